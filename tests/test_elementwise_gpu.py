"""GPU parity of GELU-tanh, SiLU-mul and the timestep embedding.

GELU-tanh: <= 1 ulp of the oracle, plus |x| * 2^-21 absolute.  The reference
evaluates 1 + tanh(u) in fp32, which cancels for u << 0 and carries an absolute
error of about |x| * 2^-24 there; the kernel evaluates the identical
x * sigmoid(2u) without that cancellation, so in the far negative tail the two
differ by the reference's own rounding, not by ulps of the (tiny) result.
SiLU-mul: <= 1 ulp.  Timestep embedding (fp32 out): |diff| <= 2e-4 -- exp, sin
and cos of two different math libraries may differ by 1-2 fp32 ulp, and the
argument t * freq (t up to 1000 rad) amplifies that in absolute terms.
"""
import pytest
import torch

from conftest import assert_guard_intact, assert_ulp_close, guarded_empty
from oracle import ops

pytestmark = pytest.mark.gpu


def rand(shape, dt, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g)).to(dt)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(10800, 12288), (6, 1024), (1, 7), (0, 8), (3, 1001)])
def test_gelu_tanh(jo, dev, dt, shape):
    x = rand(shape, dt, 1, 3.0)
    if x.numel() > 16:
        x.view(-1)[:16] = torch.tensor([0.0, -0.0, 1e-30, -1e-30, 5.0, -5.0, 8.0, -8.0, 10.0, -10.0, 30.0, -30.0,
                                        100.0, -100.0, 0.5, -0.5]).to(dt)
    out = jo.gelu_tanh(x.to(dev))
    ref = ops.gelu_tanh(x)
    bits = 23 if dt == torch.float32 else (10 if dt == torch.float16 else 7)
    tol = 64.0 if dt == torch.float32 else 1.0
    assert_ulp_close(out, ref, tol, floor=2.0 ** -126, atol=x.float().abs() * 2.0 ** -21,
                     what=f"gelu {dt} {shape} ({bits}-bit mantissa)")


def test_gelu_golden(jo, dev, golden):
    c = golden["gelu_tanh"]
    out = jo.gelu_tanh(c["x"].to(dev))
    assert_ulp_close(out, c["out"], 1.0, floor=2.0 ** -126, atol=c["x"].float().abs() * 2.0 ** -21, what="golden")


def test_gelu_unaligned_tail(jo, dev):
    base = rand((1, 4099), torch.bfloat16, 2, 2.0).to(dev)
    x = base[:, 3:]  # 6-byte offset: scalar path
    out = jo.gelu_tanh(x)
    ref = ops.gelu_tanh(x.cpu())
    assert_ulp_close(out, ref, 1.0, floor=2.0 ** -126, atol=x.cpu().float().abs() * 2.0 ** -21, what="unaligned")


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N", [(10800, 8192), (3, 100), (1, 8)])
def test_silu_mul_halves(jo, dev, dt, M, N):
    ab = rand((M, 2 * N), dt, 3, 2.0)
    a, b = ab[:, :N], ab[:, N:]
    g = ab.to(dev)
    out = jo.silu_mul(g[:, :N], g[:, N:])
    assert_ulp_close(out, ops.silu_mul(a, b), 1.0, what=f"silu_mul {dt} {M}x{N}")


def test_silu_mul_cabi_guarded(cabi, dev):
    M, N = 257, 4096
    a, b = rand((M, N), torch.bfloat16, 4).to(dev), rand((M, N), torch.bfloat16, 5).to(dev)
    buf, out = guarded_empty(M * N, torch.bfloat16, dev)
    cabi.call("jo_silu_mul", out.data_ptr(), N, a.data_ptr(), N, b.data_ptr(), N, M, N, cabi.JO_BF16, cabi.stream())
    torch.cuda.synchronize()
    assert_guard_intact(buf)
    assert_ulp_close(out.view(M, N), ops.silu_mul(a.cpu(), b.cpu()), 1.0, what="silu cabi")


@pytest.mark.parametrize("flip", [True, False])
@pytest.mark.parametrize("dim,shift", [(256, 0.0), (320, 1.0), (7, 0.0)])
def test_timestep_embedding(jo, dev, flip, dim, shift):
    g = torch.Generator().manual_seed(6)
    t = torch.rand(64, generator=g) * 1000.0
    t[0] = 0.0
    t[1] = 999.0
    out = jo.timestep_embedding(t.to(dev), dim, flip, shift, 1.0, 10000.0)
    ref = ops.timestep_embedding(t, dim, flip, shift, 1.0, 10000.0)
    # Error bound, elementwise.  The exponent (-ln P * i) / (half - shift) is the same
    # IEEE fp32 product and quotient on both sides; exp differs by <= 2 + 1 ulp (CUDA expf,
    # the CPU's exp), so f = exp(.) by <= 3 * 2^-24 relative, and the argument t * f (one
    # more rounding each) by <= |t f| * 2^-22; sin / cos add <= 2 + 1 ulp of a value in
    # [-1, 1] (<= 3 * 2^-24) and move by at most the argument's change.  Asserted with a
    # factor-2 margin: |diff| <= |t f| * 2^-21 + 2^-21.
    half = dim // 2
    f = torch.exp(-torch.log(torch.tensor(10000.0)) * torch.arange(half, dtype=torch.float32) / (half - shift))
    arg = (t[:, None] * f[None, :]).abs()
    bound = arg * 2.0 ** -21 + 2.0 ** -21
    bound = torch.cat([bound, bound], dim=1)
    if dim % 2:
        bound = torch.nn.functional.pad(bound, (0, 1))
    diff = (out.cpu() - ref).abs()
    assert (diff <= bound).all(), f"max excess {(diff - bound).max().item():.3e}"
    # frequency 0 is exact: cos(t) / sin(t) of the timestep itself
    assert (out.cpu()[:, 0 if flip else dim // 2] - torch.cos(t)).abs().max().item() <= 1e-6
