"""GPU parity of the timestep conditioning MLP (jo_timestep_mlp) against the oracle.

Stage by stage on the GPU's own stage inputs (the two intermediates come back in
the caller's scratch): each Linear output within 1 bf16 ulp (fp32 accumulation
order differs); a SiLU stage within 2 (the Linear's 1-ulp flip passes through SiLU,
slope <= 1.1, before the second rounding).  The first stage's input is the sinusoid the kernel
computes in its prologue with the arithmetic of jo_timestep_embedding, so that op's
output (rounded to bf16) is the stage input; it is itself checked against the oracle
sinusoid (|diff| <= 2e-4, CUDA vs CPU sin/cos/exp).  End to end: relative Frobenius
error <= 1e-2.
"""
import pytest
import torch

from conftest import assert_ulp_close
from oracle import ops

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def weights(freq, dim, proj, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    w = lambda n, k: (torch.randn(n, k, generator=g) / k ** 0.5).to(BF)
    b = lambda n: (0.1 * torch.randn(n, generator=g)).to(BF) if bias else None
    return w(dim, freq), b(dim), w(dim, dim), b(dim), w(proj, dim), b(proj)


def run_cabi(dev, t, ws, max_period=10000.0):
    from joyomni_ops import cabi

    w1, b1, w2, b2, w3, b3 = [None if x is None else x.to(dev) for x in ws]
    B, dim, freq, proj = t.shape[0], w1.shape[0], w1.shape[1], w3.shape[0]
    vec = torch.empty(B, proj, dtype=BF, device=dev)
    scratch = torch.empty(2, B, dim, dtype=BF, device=dev)
    p = lambda x: 0 if x is None else x.data_ptr()
    tg = t.float().to(dev)
    cabi.call("jo_timestep_mlp", vec.data_ptr(), tg.data_ptr(), B, p(w1), p(b1), freq, dim, p(w2), p(b2), p(w3),
              p(b3), proj, scratch.data_ptr(), scratch.numel() * 2, max_period, cabi.stream())
    torch.cuda.synchronize()
    return vec.cpu(), scratch[0].cpu(), scratch[1].cpu()


@pytest.mark.parametrize("B,freq,dim,proj,bias", [(1, 256, 3072, 18432, True), (2, 256, 3072, 18432, True),
                                                  (3, 256, 512, 1024, False), (9, 128, 264, 520, True),
                                                  (16, 256, 4096, 1032, True)])
def test_timestep_mlp(dev, B, freq, dim, proj, bias):
    g = torch.Generator().manual_seed(B + dim)
    t = torch.rand(B, generator=g) * 1000.0
    ws = weights(freq, dim, proj, 7 + B, bias)
    w1, b1, w2, b2, w3, b3 = ws
    vec, s1, s2 = run_cabi(dev, t, ws)
    rvec, rs1, rs2 = ops.timestep_mlp(t, *ws)
    from joyomni_ops import cabi

    e32 = torch.empty(B, freq, dtype=torch.float32, device=dev)
    tg = t.float().to(dev)
    cabi.call("jo_timestep_embedding", e32.data_ptr(), tg.data_ptr(), B, freq, 1, 0.0, 1.0, 10000.0, cabi.stream())
    # the sinusoid itself: |diff| <= 2e-4 before rounding (two math libraries; t up
    # to 1000 rad amplifies a 1-ulp exp difference), as in test_timestep_embedding
    assert (e32.cpu() - ops.timestep_embedding(t, freq)).abs().max().item() <= 2e-4
    e = e32.cpu().to(BF)
    assert_ulp_close(s1, ops.silu_bf16(ops.linear_bf16(e, w1, b1)), 2.0, what="s1 = silu(linear_1(e))")
    assert_ulp_close(s2, ops.silu_bf16(ops.linear_bf16(s1, w2, b2)), 2.0, what="s2 = silu(linear_2(s1))")
    assert_ulp_close(vec, ops.linear_bf16(s2, w3, b3), 1.0, what="vec = time_proj(s2)")
    rel = ((vec.float() - rvec.float()).norm() / rvec.float().norm()).item()
    assert rel < 1e-2, f"end to end rel err {rel}"


def test_timestep_mlp_torch_op(jo, dev):
    t = torch.tensor([0.0, 999.5], device=dev)
    ws = [None if x is None else x.to(dev) for x in weights(256, 3072, 18432, 3)]
    vec, s2 = jo.timestep_mlp(t, *ws)
    rvec, _, rs2 = ops.timestep_mlp(t.cpu(), *[None if x is None else x.cpu() for x in ws])
    assert vec.shape == (2, 18432) and s2.shape == (2, 3072)
    rel = ((vec.float().cpu() - rvec.float()).norm() / rvec.float().norm()).item()
    assert rel < 1e-2


def test_timestep_mlp_rejects(dev):
    from joyomni_ops import cabi

    ws = [x.to(dev) for x in weights(256, 512, 1024, 1)]
    t = torch.zeros(4, device=dev)
    vec = torch.empty(4, 1024, dtype=BF, device=dev)
    small = torch.empty(100, dtype=BF, device=dev)
    st = cabi.status_of("jo_timestep_mlp", vec.data_ptr(), t.data_ptr(), 4, ws[0].data_ptr(), ws[1].data_ptr(), 256,
                        512, ws[2].data_ptr(), ws[3].data_ptr(), ws[4].data_ptr(), ws[5].data_ptr(), 1024,
                        small.data_ptr(), 200, 10000.0, cabi.stream())
    assert st == cabi.JO_ERR_SHAPE
    assert "scratch" in cabi.last_error()


@pytest.mark.parametrize("B,n_tables", [(1, 80), (2, 3), (1, 0)])
def test_timestep_mlp_modulate(jo, dev, B, n_tables):
    """The ModulateWan add (dit.py:103-116: modulate_table + vec in bf16) folded into
    time_proj's epilogue: vec equals the plain MLP's bit for bit, and every block's
    modulation rows equal bf16(table + vec) bit for bit."""
    D = 3072
    t = (torch.rand(B, generator=torch.Generator().manual_seed(40 + B)) * 1000.0).to(dev)
    ws = [None if x is None else x.to(dev) for x in weights(256, D, 6 * D, 41)]
    g = torch.Generator().manual_seed(42)
    tables = (torch.randn(n_tables, 6, D, generator=g) / D ** 0.5).to(BF).to(dev)
    vec, mods = jo.timestep_mlp_modulate(t, *ws, tables)
    want_vec, _ = jo.timestep_mlp(t, *ws)
    assert torch.equal(vec, want_vec)
    assert mods.shape == (n_tables, B, 6 * D)
    # the module's own arithmetic on the bf16 time_proj output (dit.py:115)
    want = tables.view(n_tables, 1, 6 * D) + vec.view(1, B, 6 * D)
    assert torch.equal(mods, want)
