"""The torch boundary refuses misplaced operands before any kernel runs.

Every tensor operand of every op must be a CUDA tensor on the op's device; a host
tensor (or another GPU's) passed as a scale, weight, table, gate or output must
raise RuntimeError in the shim, never reach a kernel as a foreign pointer.  The
launch counter of the C ABI shows that nothing was launched.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
FP8 = torch.float8_e4m3fn


def _cases(jo, dev, other):
    """(name, thunk) pairs; `other` is where the misplaced operand lives."""
    M, N, H, D = 64, 256, 2, 128
    x = torch.randn(M, N, device=dev).to(BF)
    w = torch.ones(N, dtype=BF, device=dev)
    mod = torch.zeros(1, N, dtype=BF, device=dev)
    aq = torch.zeros(M, N, dtype=FP8, device=dev)
    bq = torch.zeros(N, 128, dtype=FP8, device=dev).t()
    sa, sb = torch.ones(M, 1, device=dev), torch.ones(1, 128, device=dev)
    qkv = torch.randn(16, 3 * H * D, device=dev).to(BF)
    hw = torch.ones(D, dtype=BF, device=dev)
    tab = torch.ones(16, D // 2, dtype=BF, device=dev)
    q4 = torch.randn(1, 16, H, D, device=dev).to(BF)
    ftab = torch.ones(16, D, device=dev)
    o = lambda t: t.to(other)
    return [
        ("rmsnorm weight", lambda: jo.rmsnorm(x, o(w), 1e-6)),
        ("norm scale", lambda: jo.fused_norm_scale_shift(x, None, None, o(mod), mod, "layer")),
        ("norm gamma", lambda: jo.fused_norm_scale_shift(x, o(w), None, mod, mod, "layer")),
        ("quant output_s", lambda: jo.sgl_per_token_quant_fp8(x, torch.empty(M, N, dtype=FP8, device=dev),
                                                              o(torch.empty(M, 1)))),
        ("gemm scales_a", lambda: jo.fp8_scaled_mm(aq, bq, o(sa), sb, BF, None)),
        ("gemm scales_b", lambda: jo.fp8_scaled_mm(aq, bq, sa, o(sb), BF, None)),
        ("gemm bias", lambda: jo.fp8_scaled_mm(aq, bq, sa, sb, BF, o(torch.zeros(128, dtype=BF)))),
        ("gemm residual", lambda: jo.fp8_scaled_mm_gated_residual(aq, bq, sa, sb, BF, None,
                                                                  o(torch.zeros(M, 128, dtype=BF)),
                                                                  torch.ones(128, dtype=BF, device=dev))),
        ("pack cos", lambda: jo.qkv_norm_rope_pack(qkv, H, hw, hw, o(tab), tab)),
        ("pack q_weight", lambda: jo.qkv_norm_rope_pack(qkv, H, o(hw), hw, tab, tab)),
        ("paired sin", lambda: jo.fused_qk_norm_rope_3d_paired(q4.view(1, 32, D).clone(), q4.view(1, 32, D).clone(),
                                                                16, H, 1e-6, hw, hw, tab, o(tab))),
        ("joint txt weight", lambda: jo.fused_joint_qkv_pack(q4, q4, q4, q4, q4, q4, None, None, o(hw), hw)),
        ("cached cos", lambda: jo.fused_cached_kv_pack(q4, q4, None, None, o(ftab), ftab)),
        ("gated residual gate", lambda: jo.gated_residual(x, x, o(w))),
        ("gated ln scale", lambda: jo.gated_residual_norm_scale_shift(x, x, w, o(mod), mod)),
        ("silu_mul b", lambda: jo.silu_mul(x, o(x))),
        ("rmsnorm_quant weight", lambda: jo.rmsnorm_quant_fp8(x, o(w))),
        ("nss quant shift", lambda: jo.norm_scale_shift_quant_fp8(x, None, None, mod, o(mod))),
    ]


def test_host_operand_raises_before_launch(jo, cabi, dev):
    for name, thunk in _cases(jo, dev, "cpu"):
        n0 = cabi.launch_count()
        with pytest.raises(RuntimeError):
            thunk()
        assert cabi.launch_count() == n0, f"{name}: a kernel was launched"
    torch.cuda.synchronize()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_other_device_operand_raises_before_launch(jo, cabi, dev):
    for name, thunk in _cases(jo, dev, torch.device("cuda", 1)):
        n0 = cabi.launch_count()
        with pytest.raises(RuntimeError, match="op runs on|must be a CUDA tensor"):
            thunk()
        assert cabi.launch_count() == n0, f"{name}: a kernel was launched"
    torch.cuda.synchronize()
