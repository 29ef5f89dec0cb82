"""GPU parity of the tcgen05 FP8 GEMM (jo_fp8_scaled_mm / joyomni_ops.fp8_scaled_mm).

Oracle: oracle.ops.fp8_scaled_mm (float64 dot products of the e4m3 operands,
then the reference EVT order (acc * sB) * sA (+ bias) in fp32, one rounding).
Gate: per-element |D - ref| <= 2 ulp(out dtype, |ref|) + 2^-12 * rms(ref); the
north-star gate (relative Frobenius error <= 2e-2) is asserted too.  The
BASELINE shapes check every row against the CPU oracle (in blocks of rows) and
the whole matrix against torch._scaled_mm on the GPU as well.
"""
import pytest
import torch

from conftest import assert_guard_intact, assert_ulp_close, guarded_empty
from oracle import ops

pytestmark = pytest.mark.gpu
FP8 = torch.float8_e4m3fn


def operands(M, N, K, seed, dt=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dt)
    w = (0.02 * torch.randn(N, K, generator=g)).to(dt)
    aq, sa = ops.per_token_quant_fp8(x)                  # A [M, K] row-major, sA [M, 1]
    bq, sb = ops.quantize_weight_per_channel(w)          # B [K, N] column-major, sB [1, N]
    return aq, sa, bq, sb


def check(out, ref, what):
    o, r = out.float().cpu(), ref.float().cpu()
    bits = 7 if ref.dtype == torch.bfloat16 else 10
    rms = r.pow(2).mean().sqrt().item() if r.numel() else 0.0
    ulp = torch.pow(2.0, torch.floor(torch.log2(r.abs().clamp_min(1e-30))) - bits)
    allowed = 2 * ulp + rms * 2.0 ** -12
    bad = (o - r).abs() > allowed
    assert not bad.any(), (f"{what}: {bad.sum().item()} of {o.numel()} off; max |d| "
                           f"{(o - r).abs().max().item():.3e}, rms {rms:.3e}")
    rel = ((o - r).norm() / r.norm().clamp_min(1e-30)).item()
    assert rel <= 2e-2, f"{what}: rel err {rel}"
    return rel


def run(jo, dev, aq, sa, bq, sb, bias=None, out_dtype=torch.bfloat16):
    return jo.fp8_scaled_mm(aq.to(dev), bq.to(dev), sa.to(dev), sb.to(dev), out_dtype,
                            bias.to(dev) if bias is not None else None)


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (1, 8, 16), (67, 264, 48), (129, 512, 3072 + 16),
                                   (300, 1000, 256), (256, 256, 4096)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_gemm_small(jo, dev, M, N, K, out_dtype):
    aq, sa, bq, sb = operands(M, N, K, M + N + K)
    d = run(jo, dev, aq, sa, bq, sb, out_dtype=out_dtype)
    check(d, ops.fp8_scaled_mm(aq, bq, sa, sb, None, out_dtype), f"{M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(200, 264, 512), (10800, 256, 3072)])
def test_gemm_bias(jo, dev, M, N, K):
    aq, sa, bq, sb = operands(M, N, K, 5)
    bias = (0.1 * torch.randn(N, generator=torch.Generator().manual_seed(6))).to(torch.bfloat16)
    d = run(jo, dev, aq, sa, bq, sb, bias)
    check(d, ops.fp8_scaled_mm(aq, bq, sa, sb, bias, torch.bfloat16), "bias")


@pytest.mark.parametrize("M,N,K", [(10800, 9216, 3072), (10800, 12288, 3072), (4096, 4096, 4096)])
def test_gemm_baseline_shapes(jo, dev, M, N, K):
    """Benchmark config 3 (QKV and MLP-up projections) and the reference bench shape."""
    aq, sa, bq, sb = operands(M, N, K, 7)
    ag, bg, sag, sbg = aq.to(dev), bq.to(dev), sa.to(dev), sb.to(dev)
    d = jo.fp8_scaled_mm(ag, bg, sag, sbg, torch.bfloat16, None).cpu()
    # every row against the CPU oracle, a block of rows at a time
    for r0 in range(0, M, 1800):
        r1 = min(M, r0 + 1800)
        ref = ops.fp8_scaled_mm(aq[r0:r1], bq, sa[r0:r1], sb, None, torch.bfloat16)
        check(d[r0:r1], ref, f"{M}x{N}x{K} rows {r0}:{r1}")
    d = d.to(dev)
    # whole matrix against the library scaled GEMM (cross-check only)
    lib = torch._scaled_mm(ag, bg, scale_a=sag, scale_b=sbg, out_dtype=torch.bfloat16)
    rel = ((d.float() - lib.float()).norm() / lib.float().norm()).item()
    assert rel < 5e-3, f"vs torch._scaled_mm: rel {rel}"


def test_gemm_reference_bench_quant(jo, dev):
    """joyomni_ops/tests/test_bench.py:160-200: weight quantised with the per-token
    op on [N, K] and passed transposed (column-major)."""
    M = N = K = 1024
    g = torch.Generator().manual_seed(9)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    w = torch.randn(N, K, generator=g).to(torch.bfloat16).to(dev)
    wq = torch.empty(N, K, device=dev, dtype=FP8)
    wsc = torch.empty(N, device=dev, dtype=torch.float32)
    jo.sgl_per_token_quant_fp8(w, wq, wsc)
    xq = torch.empty(M, K, device=dev, dtype=FP8)
    xsc = torch.empty(M, device=dev, dtype=torch.float32)
    jo.sgl_per_token_quant_fp8(x, xq, xsc)
    d = jo.fp8_scaled_mm(xq, wq.t(), xsc, wsc, torch.bfloat16, None)
    ref = ops.fp8_scaled_mm(xq.cpu(), wq.t().cpu(), xsc.cpu(), wsc.cpu(), None, torch.bfloat16)
    check(d, ref, "bench-style")
    # the inherent FP8 quantisation loss vs the bf16 GEMM is a few percent (README: 3.7 %)
    full = (x.float() @ w.float().t())
    rel = ((d.float() - full).norm() / full.norm()).item()
    assert rel < 0.06


def test_gemm_cabi_guarded(cabi, dev):
    M, N, K = 131, 264, 256
    aq, sa, bq, sb = operands(M, N, K, 11)
    ag, bg, sag, sbg = aq.to(dev), bq.to(dev), sa.to(dev).reshape(-1), sb.to(dev).reshape(-1)
    LDD = N + 8
    buf, mid = guarded_empty(M * LDD, torch.bfloat16, dev)
    cabi.call("jo_fp8_scaled_mm", mid.data_ptr(), LDD, ag.data_ptr(), K, bg.data_ptr(), K, sag.data_ptr(),
              sbg.data_ptr(), None, M, N, K, cabi.JO_BF16, cabi.stream())
    torch.cuda.synchronize()
    assert_guard_intact(buf)
    check(mid.view(M, LDD)[:, :N], ops.fp8_scaled_mm(aq, bq, sa, sb, None, torch.bfloat16), "guarded")
    assert cabi.device_fault_count() == 0


def test_gemm_rejects(jo, dev, cabi):
    a = torch.zeros(64, 24, dtype=FP8, device=dev)
    b = torch.zeros(24, 64, dtype=FP8, device=dev).t().contiguous().t()
    s = torch.ones(64, device=dev)
    with pytest.raises(RuntimeError, match="16 bytes"):
        jo.fp8_scaled_mm(a, b, s, s, torch.bfloat16, None)
    st = cabi.status_of("jo_fp8_scaled_mm", 0, 64, 0, 32, 0, 32, 0, 0, None, 64, 64, 32, cabi.JO_BF16, None)
    assert st == cabi.JO_ERR_INVALID


@pytest.mark.parametrize("M,N,K,bias", [(10800, 3072, 12288, True), (200, 264, 512, False), (100, 512, 256, True),
                                        (512, 3072, 12288, True)])
def test_gemm_gated_residual(jo, dev, M, N, K, bias):
    """Down projection + gated residual in the GEMM epilogue (dit.py:536-538)."""
    aq, sa, bq, sb = operands(M, N, K, 11)
    g = torch.Generator().manual_seed(12)
    b = (0.1 * torch.randn(N, generator=g)).to(torch.bfloat16) if bias else None
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    gate = (0.1 * torch.randn(1, N, generator=g)).to(torch.bfloat16)
    d = jo.fp8_scaled_mm_gated_residual(aq.to(dev), bq.to(dev), sa.to(dev), sb.to(dev), torch.bfloat16,
                                        None if b is None else b.to(dev), res.to(dev), gate.to(dev))
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(13))[:160]
    rows = torch.cat([rows, torch.tensor([0, M - 1])])
    ref = ops.fp8_scaled_mm_gated_residual(aq[rows], bq, sa[rows], sb, b, res[rows], gate)
    # the product enters in fp32 (no intermediate rounding): per element <= 2 ulp of the
    # result plus |gate| * 2^-12 * rms(product) for the GEMM's accumulation order
    prod = ops.fp8_scaled_mm(aq[rows], bq, sa[rows], sb, b, torch.float32)
    atol = gate.float().abs().reshape(1, -1) * prod.pow(2).mean().sqrt() * 2.0 ** -12
    assert_ulp_close(d.cpu()[rows], ref, 2.0, what="gated residual GEMM", atol=atol.expand_as(ref))
    # against the unfused chain: GEMM rounded to bf16, then addcmul
    unfused = ops.gated_residual(res[rows], ops.fp8_scaled_mm(aq[rows], bq, sa[rows], sb, b, torch.bfloat16), gate)
    rel = ((d.cpu()[rows].float() - unfused.float()).norm() / unfused.float().norm()).item()
    assert rel < 1e-3


def test_gemm_gated_residual_in_place(jo, dev):
    """D may alias the residual (same rows and stride)."""
    from joyomni_ops import cabi

    M, N, K = 300, 512, 256
    aq, sa, bq, sb = operands(M, N, K, 14)
    res = torch.randn(M, N, generator=torch.Generator().manual_seed(15)).to(torch.bfloat16)
    gate = torch.full((N,), 0.5).to(torch.bfloat16)
    ref = ops.fp8_scaled_mm_gated_residual(aq, bq, sa, sb, None, res, gate)
    ag, bg, sag, sbg, rg, gg = aq.to(dev), bq.to(dev), sa.to(dev), sb.to(dev), res.to(dev), gate.to(dev)
    cabi.call("jo_fp8_scaled_mm_gated_residual", rg.data_ptr(), N, ag.data_ptr(), K, bg.data_ptr(), bg.stride(1),
              sag.data_ptr(), sbg.data_ptr(), 0, rg.data_ptr(), N, gg.data_ptr(), M, N, K, cabi.JO_BF16,
              cabi.stream())
    torch.cuda.synchronize()
    assert_ulp_close(rg.cpu(), ref, 2.0, what="in place", atol=torch.full((M, N), 2.0 ** -10))


# ------------------------------------------------------------------ fc1 -> GELU -> FP8
@pytest.mark.parametrize("M,N,K,bias,dt", [(10800, 12288, 3072, True, torch.bfloat16),
                                           (512, 12288, 3072, True, torch.bfloat16),
                                           (100, 520, 256, False, torch.bfloat16),
                                           (300, 264, 512, True, torch.float16),
                                           (129, 8, 16, False, torch.bfloat16)])
def test_gemm_gelu_quant(jo, dev, M, N, K, bias, dt):
    """The MLP's fc1 -> GELU-tanh -> per-token FP8 in one op (GELU and the row amax in the GEMM
    epilogue, then a quantisation pass) equals this library's unfused chain bit for bit:
    fp8_scaled_mm, then gelu_quant_fp8.  Sizes: the BASELINE fc1 [10800, 3072] x [3072, 12288],
    the single-CTA kernel (M <= 128), N not a multiple of the 256-column tile, fp16."""
    aq, sa, bq, sb = operands(M, N, K, 21)
    g = torch.Generator().manual_seed(22)
    b = (0.1 * torch.randn(N, generator=g)).to(dt) if bias else None
    ag, bg, sag, sbg = aq.to(dev), bq.to(dev), sa.to(dev), sb.to(dev)
    bgpu = None if b is None else b.to(dev)
    q, s = jo.fp8_scaled_mm_gelu_quant(ag, bg, sag, sbg, dt, bgpu)
    up = jo.fp8_scaled_mm(ag, bg, sag, sbg, dt, bgpu)
    q2, s2 = jo.gelu_quant_fp8(up)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8)), "quantised GELU differs from the unfused chain"
    assert torch.equal(s, s2), "row scales differ from the unfused chain"
    # against the oracle (fc1 in float64 dot products, torch's GELU), dequantised, on sampled rows
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(23))[:64]
    rows = torch.cat([rows, torch.tensor([0, M - 1])])
    ref = ops.gelu_tanh(ops.fp8_scaled_mm(aq[rows], bq, sa[rows], sb, b, dt)).float()
    got = q.cpu()[rows].float() * s.cpu()[rows]
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert rel < 0.05, rel  # e4m3 keeps 3 mantissa bits: <= 2^-4 relative per element


def test_gemm_gelu_quant_cabi(cabi, dev):
    """The C ABI: guarded outputs, the GELU left in the caller's y workspace, and the amax
    workspace reset on the stream (it starts as garbage here)."""
    import joyomni_ops as jo

    M, N, K = 260, 264, 256
    aq, sa, bq, sb = operands(M, N, K, 24)
    ag, bg, sag, sbg = aq.to(dev), bq.to(dev), sa.to(dev).reshape(-1), sb.to(dev).reshape(-1)
    LDQ, LDY = N + 8, N + 16
    qbuf, qmid = guarded_empty(M * LDQ, torch.uint8, dev)
    sbuf, smid = guarded_empty(M, torch.float32, dev)
    y = torch.empty(M, LDY, dtype=torch.bfloat16, device=dev)
    amax = torch.full((M,), 0x7F7F7F7F, dtype=torch.int32, device=dev)
    cabi.call("jo_fp8_scaled_mm_gelu_quant", qmid.data_ptr(), LDQ, smid.data_ptr(), y.data_ptr(), LDY,
              amax.data_ptr(), ag.data_ptr(), K, bg.data_ptr(), K, sag.data_ptr(), sbg.data_ptr(), None, M, N, K,
              cabi.JO_BF16, cabi.stream())
    torch.cuda.synchronize()
    assert_guard_intact(qbuf)
    assert_guard_intact(sbuf)
    up = jo.fp8_scaled_mm(ag, bg, sag.reshape(-1, 1), sbg.reshape(1, -1), torch.bfloat16, None)
    gelu = jo.gelu_tanh(up)
    assert torch.equal(y[:, :N], gelu)
    q2, s2 = jo.gelu_quant_fp8(up)  # GELU -> FP8 of the GEMM output
    assert torch.equal(qmid.view(M, LDQ)[:, :N], q2.view(torch.uint8))
    assert torch.equal(smid, s2.reshape(-1))
    assert cabi.device_fault_count() == 0


def test_gemm_gelu_quant_rejects(cabi, dev):
    a = torch.zeros(64, 32, dtype=FP8, device=dev)
    w = torch.zeros(64, 32, dtype=FP8, device=dev)
    s = torch.ones(64, device=dev)
    q = torch.empty(64, 64, dtype=torch.uint8, device=dev)
    y = torch.empty(64, 64, dtype=torch.bfloat16, device=dev)
    am = torch.empty(64, dtype=torch.int32, device=dev)
    args = lambda n, ldq, ws: (q.data_ptr(), ldq, s.data_ptr(), y.data_ptr(), 64, ws, a.data_ptr(), 32,
                               w.data_ptr(), 32, s.data_ptr(), s.data_ptr(), None, 64, n, 32, cabi.JO_BF16, None)
    assert cabi.status_of("jo_fp8_scaled_mm_gelu_quant", *args(0, 64, am.data_ptr())) == cabi.JO_ERR_SHAPE
    assert cabi.status_of("jo_fp8_scaled_mm_gelu_quant", *args(64, 64, None)) == cabi.JO_ERR_INVALID
    assert cabi.status_of("jo_fp8_scaled_mm_gelu_quant", *args(64, 68, am.data_ptr())) == cabi.JO_ERR_ALIGN
    torch.cuda.synchronize()
