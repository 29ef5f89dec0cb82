"""GPU parity of the row kernels against the CPU oracle (tolerances in the asserts).

bf16/fp16 outputs: <= 1 ulp of the oracle value (ulp taken at max(|ref|, 2^-10)
so cancellation to tiny values is judged against the O(1) terms); fp32
outputs: <= 64 fp32 ulps of max(|ref|, 0.25) (reduction order; the modulated
terms are O(1) and cancel).  FP8 bytes and scales: bit-exact.
"""
import pytest
import torch

from conftest import assert_guard_intact, assert_ulp_close, guarded_empty
from oracle import ops

pytestmark = pytest.mark.gpu

SHAPES = [(3600, 3072), (1, 3072), (0, 3072), (37, 136), (5, 12288), (9, 100), (4, 24576), (3, 40000),
          (11, 2048), (13, 1536), (150, 1024)]  # row groups of 1, 2 and 4 warps
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def ulps(dt):
    return 64.0 if dt == torch.float32 else 1.0


def floor_for(dt):
    return 0.25 if dt == torch.float32 else 2.0 ** -10


def rand(shape, dt, seed, scale=1.0, mean=0.0):
    g = torch.Generator().manual_seed(seed)
    return (mean + scale * torch.randn(*shape, generator=g)).to(dt)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_rmsnorm(jo, dev, dt, shape):
    M, N = shape
    x = rand(shape, dt, 1)
    w = rand((N,), dt, 2, 0.02, 1.0)
    out = jo.rmsnorm(x.to(dev), w.to(dev), 1e-6)
    assert_ulp_close(out, ops.rmsnorm(x, w, 1e-6), ulps(dt), floor_for(dt), what=f"rmsnorm {dt} {shape}")


def test_rmsnorm_cabi_strided_guarded(cabi, dev):
    # rows of a wider tensor in, rows of a wider buffer out; canaries around it
    M, N, XS, OS = 300, 3072, 3072 + 64, 3072 + 8
    xw = rand((M, XS), torch.bfloat16, 3)
    w = rand((N,), torch.bfloat16, 4, 0.02, 1.0)
    xg, wg = xw.to(dev), w.to(dev)
    buf, mid = guarded_empty(M * OS, torch.bfloat16, dev)
    cabi.call("jo_rmsnorm", mid.data_ptr(), OS, xg.data_ptr(), XS, wg.data_ptr(), M, N, cabi.JO_BF16, 1e-6,
              cabi.stream())
    torch.cuda.synchronize()
    assert_guard_intact(buf)
    out = mid.view(M, OS)[:, :N]
    assert_ulp_close(out, ops.rmsnorm(xw[:, :N], w, 1e-6), 1.0, what="rmsnorm strided")


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("norm", ["layer", "rms"])
@pytest.mark.parametrize("per_row", [False, True])
@pytest.mark.parametrize("affine", [False, True])
@pytest.mark.parametrize("shape", [(10800, 3072), (33, 4096), (7, 12288), (5, 64)])
def test_norm_scale_shift(jo, dev, dt, norm, per_row, affine, shape):
    M, N = shape
    x = rand(shape, dt, 10)
    mr = M if per_row else 1
    scale = rand((mr, N), dt, 11, 0.1)
    shift = rand((mr, N), dt, 12, 0.1)
    gamma = rand((N,), dt, 13, 0.5, 1.0) if affine else None
    beta = rand((N,), dt, 14, 0.5) if (affine and norm == "layer") else None
    g = lambda t: t.to(dev) if t is not None else None
    out = jo.fused_norm_scale_shift(g(x), g(gamma), g(beta), g(scale), g(shift), norm, 1e-6)
    ref = ops.norm_scale_shift(x, gamma, beta, scale, shift, norm, 1e-6)
    assert_ulp_close(out, ref, ulps(dt), floor_for(dt), what=f"norm_scale_shift {norm} {dt} {shape}")


def test_norm_scale_shift_rejects(jo, dev):
    x = torch.randn(4, 64, device=dev, dtype=torch.bfloat16)
    s = torch.randn(2, 64, device=dev, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="scale/shift rows"):
        jo.fused_norm_scale_shift(x, None, None, s, s, "layer", 1e-6)
    s1 = s[:1]
    with pytest.raises(RuntimeError, match="norm_type"):
        jo.fused_norm_scale_shift(x, None, None, s1, s1, "bogus", 1e-6)
    with pytest.raises(RuntimeError, match="divisible by 4"):
        jo.fused_norm_scale_shift(x[:, :62], None, None, s1[:, :62], s1[:, :62], "layer", 1e-6)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(10800, 3072), (1, 3072), (17, 200), (5, 12288)])
def test_gated_residual(jo, dev, dt, shape):
    M, N = shape
    res, x = rand(shape, dt, 20), rand(shape, dt, 21)
    gate = rand((1, N), dt, 22, 0.1)
    out = jo.gated_residual(res.to(dev), x.to(dev), gate.to(dev))
    assert_ulp_close(out, ops.gated_residual(res, x, gate), 1.0, what=f"gated_residual {shape}")
    gate_rows = rand((M, N), dt, 23, 0.1)
    out = jo.gated_residual(res.to(dev), x.to(dev), gate_rows.to(dev))
    assert_ulp_close(out, ops.gated_residual(res, x, gate_rows), 1.0, what="gated_residual per-row gate")


@pytest.mark.parametrize("norm", ["layer", "rms"])
@pytest.mark.parametrize("shape", [(10800, 3072), (3, 3072), (9, 100), (4, 12288)])
def test_gated_residual_norm_scale_shift(jo, dev, norm, shape):
    M, N = shape
    dt = torch.bfloat16
    res, x = rand(shape, dt, 30), rand(shape, dt, 31)
    gate = rand((1, N), dt, 32, 0.1)
    scale, shift = rand((1, N), dt, 33, 0.1), rand((1, N), dt, 34, 0.1)
    h, y = jo.gated_residual_norm_scale_shift(res.to(dev), x.to(dev), gate.to(dev), scale.to(dev), shift.to(dev),
                                              norm, 1e-6)
    assert_ulp_close(h, ops.gated_residual(res, x, gate), 1.0, what="h")
    # y is Norm(h) of the kernel's own h (h itself is checked above)
    y_ref = ops.norm_scale_shift(h.cpu(), None, None, scale, shift, norm, 1e-6)
    assert_ulp_close(y, y_ref, 1.0, what=f"y {norm} {shape}")


def quant_inputs(M, N, dt, seed):
    x = rand((M, N), dt, seed)
    if M > 3:
        x[0].zero_()  # zero row: scale 1e-8/448, q = 0
        x[1] *= 1e-3  # in fp16 some of these underflow to +-0: the byte keeps the sign (0x00 / 0x80)
        x[2] *= 300.0
        x[3, 5] = 448.0 * 3  # a row whose max sits far from the bulk
    if M > 4 and N > 8:
        x[4, :4] = torch.tensor([0.0, -0.0, 1.0, -1.0]).to(dt)
        x[4, 4:8] = -0.0
    return x


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(10800, 3072), (67, 4096), (1, 16), (0, 3072), (9, 100), (5, 12288), (6, 24),
                                   (19, 2048), (7, 1040)])
def test_per_token_quant_bit_exact(jo, dev, dt, shape):
    M, N = shape
    x = quant_inputs(M, N, dt, 40)
    q = torch.empty(M, N, dtype=torch.float8_e4m3fn, device=dev)
    s = torch.empty(M, 1, dtype=torch.float32, device=dev)
    jo.sgl_per_token_quant_fp8(x.to(dev), q, s)
    rq, rs = ops.per_token_quant_fp8(x)
    assert torch.equal(s.cpu(), rs), "scales differ"
    qb, rb = q.cpu().view(torch.uint8), rq.view(torch.uint8)
    if not torch.equal(qb, rb):
        i = (qb != rb).nonzero()[0].tolist()
        raise AssertionError(f"{(qb != rb).sum().item()} fp8 bytes differ; first at {i}: x={x[i[0], i[1]].item()!r} "
                             f"got {qb[i[0], i[1]].item():#04x} want {rb[i[0], i[1]].item():#04x}")


def test_per_token_quant_reference_assert(jo, dev):
    """joyomni_ops/tests/test_parity_light.py:113-133, asserted the same way.

    The reference formula is evaluated on the CPU (the oracle).  Evaluated with
    torch on the GPU instead, the same formula differs from its own CPU result
    in a few rounding-boundary elements, so that comparison is looser.
    """
    M, N = 67, 4096
    x = torch.randn(M, N, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
    x[0].zero_()
    q = torch.empty(M, N, dtype=torch.float8_e4m3fn, device=dev)
    scale = torch.empty((M, 1), device=dev, dtype=torch.float32)
    jo.sgl_per_token_quant_fp8(x.to(dev), q, scale)
    q, scale = q.cpu(), scale.cpu()

    def rel(xr):
        ref_scale = xr.abs().amax(dim=1, keepdim=True).float().clamp_min(1e-8) / 448.0
        ref_q = (xr.float() / ref_scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
        ref_scale, ref_q = ref_scale.cpu(), ref_q.cpu()
        scale_rel = ((scale - ref_scale).abs().max() / ref_scale.abs().max().clamp_min(1e-9)).item()
        q_rel = ((q.float() * scale - ref_q.float() * ref_scale).abs().mean()
                 / (ref_q.float() * ref_scale).abs().mean().clamp_min(1e-9)).item()
        return scale_rel, q_rel

    s_rel, q_rel = rel(x)
    assert s_rel == 0.0 and q_rel == 0.0  # bit-exact to the CPU reference formula
    s_rel, q_rel = rel(x.to(dev))
    assert s_rel < 1e-5 and q_rel < 1e-4


@pytest.mark.parametrize("shape", [(10800, 3072), (40, 4096), (3, 136), (2, 12288)])
def test_rmsnorm_quant_fp8(jo, dev, shape):
    M, N = shape
    x = rand(shape, torch.bfloat16, 50)
    w = rand((N,), torch.bfloat16, 51, 0.02, 1.0)
    xg, wg = x.to(dev), w.to(dev)
    q, s = jo.rmsnorm_quant_fp8(xg, wg, 1e-6)
    y_kernel = jo.rmsnorm(xg, wg, 1e-6).cpu()  # same row kernel, same bf16 intermediate
    cq, cs = ops.per_token_quant_fp8(y_kernel)
    assert torch.equal(s.cpu(), cs) and torch.equal(q.cpu().view(torch.uint8), cq.view(torch.uint8))
    # against the full oracle chain: bit-exact on every row whose bf16 intermediate matches
    y_ref = ops.rmsnorm(x, w, 1e-6)
    rq, rs = ops.rmsnorm_quant_fp8(x, w, 1e-6)
    same = (y_kernel == y_ref).all(dim=1)
    assert same.float().mean().item() > 0.5
    assert torch.equal(q.cpu()[same].view(torch.uint8), rq[same].view(torch.uint8))
    assert torch.equal(s.cpu()[same], rs[same])


@pytest.mark.parametrize("norm", ["layer", "rms"])
@pytest.mark.parametrize("shape", [(10800, 3072), (3, 4096), (5, 100)])
def test_norm_scale_shift_quant_fp8(jo, dev, norm, shape):
    M, N = shape
    x = rand(shape, torch.bfloat16, 60)
    scale, shift = rand((1, N), torch.bfloat16, 61, 0.1), rand((1, N), torch.bfloat16, 62, 0.1)
    g = lambda t: t.to(dev)
    q, s = jo.norm_scale_shift_quant_fp8(g(x), None, None, g(scale), g(shift), norm, 1e-6)
    y_kernel = jo.fused_norm_scale_shift(g(x), None, None, g(scale), g(shift), norm, 1e-6).cpu()
    cq, cs = ops.per_token_quant_fp8(y_kernel)
    assert torch.equal(s.cpu(), cs) and torch.equal(q.cpu().view(torch.uint8), cq.view(torch.uint8))
    y_ref = ops.norm_scale_shift(x, None, None, scale, shift, norm, 1e-6)
    assert_ulp_close(y_kernel, y_ref, 1.0, what="intermediate")


def test_quant_cabi_guarded(cabi, dev):
    M, N = 129, 3072
    x = quant_inputs(M, N, torch.bfloat16, 70).to(dev)
    qbuf, q = guarded_empty(M * N, torch.uint8, dev)
    sbuf, s = guarded_empty(M, torch.float32, dev)
    cabi.call("jo_per_token_quant_fp8", q.data_ptr(), N, s.data_ptr(), x.data_ptr(), N, M, N, cabi.JO_BF16,
              cabi.stream())
    torch.cuda.synchronize()
    assert_guard_intact(qbuf)
    assert_guard_intact(sbuf)
    rq, rs = ops.per_token_quant_fp8(x.cpu())
    assert torch.equal(q.view(M, N).cpu(), rq.view(torch.uint8)) and torch.equal(s.cpu(), rs.view(-1))


def test_cabi_error_paths(cabi, dev):
    x = torch.zeros(4, 64, device=dev, dtype=torch.bfloat16)
    assert cabi.status_of("jo_rmsnorm", x.data_ptr(), 64, x.data_ptr(), 64, None, 4, 64, cabi.JO_BF16, 1e-6,
                          None) == cabi.JO_ERR_INVALID
    assert cabi.status_of("jo_rmsnorm", x.data_ptr(), 64, x.data_ptr(), 64, x.data_ptr(), 4, 64, 99, 1e-6,
                          None) == cabi.JO_ERR_DTYPE
    assert cabi.status_of("jo_per_token_quant_fp8", x.data_ptr(), 64, x.data_ptr(), x.data_ptr(), 64, 4, 64,
                          cabi.JO_F32, None) == cabi.JO_ERR_DTYPE
    assert cabi.status_of("jo_rmsnorm", x.data_ptr(), 64, x.data_ptr(), 64, x.data_ptr(), -1, 64, cabi.JO_BF16,
                          1e-6, None) == cabi.JO_ERR_SHAPE
    assert "negative" in cabi.last_error()
