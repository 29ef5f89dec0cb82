"""Pin the CPU oracle against golden vectors produced by the reference's own code.

tests/golden/reference_golden.pt is written by tests/golden/make_golden.py,
which imports the reference's sgl_fused_ops.py / fp8_linear.py / rope.py by file
path and runs them.  Where the oracle restates exactly the reference function,
the match is bit-exact; where the oracle follows the reference KERNEL's rounding
(one rounding) and the golden is the reference's PyTorch path (more roundings),
the difference is bounded in bf16 ulps and both sides are checked.
"""
import torch

from conftest import assert_bf16_close
from oracle import ops


def test_rmsnorm_bit_exact(golden):
    for name in ("rmsnorm_7x3072", "rmsnorm_5x136", "rmsnorm_3x4096", "rmsnorm_qk_bf16"):
        c = golden[name]
        out = ops.rmsnorm(c["x"], c["w"], c["eps"])
        assert torch.equal(out, c["out"]), name


def test_rmsnorm_f16_f32_bit_exact(golden):
    for name in ("rmsnorm_float16", "rmsnorm_float32"):
        c = golden[name]
        out = ops.rmsnorm(c["x"], c["w"], c["eps"])
        assert out.dtype == c["out"].dtype and torch.equal(out, c["out"]), name


def test_rmsnorm_model_vs_kernel_semantics(golden):
    # The model's double-rounding RMSNorm is within 1 ulp of the single-rounding one.
    c = golden["rmsnorm_7x3072"]
    assert_bf16_close(ops.rmsnorm_model(c["x"], c["w"], c["eps"]), c["out"], 1.0, what="rmsnorm_model")


def test_layernorm_modulate(golden):
    c = golden["layernorm_modulate"]
    shim = ops.layernorm_modulate_shim(c["x"], c["shift"], c["scale"], c["eps"])
    assert torch.equal(shim, c["out"])
    x2 = c["x"].reshape(-1, 3072)
    one = ops.norm_scale_shift(x2, None, None, c["scale"], c["shift"], "layer", c["eps"])
    # single rounding vs the shim's bf16 arithmetic: the shim rounds (1 + scale)
    # to bf16 (ulp 2^-7), so the two differ by a few ulps of the O(1) terms.
    assert_bf16_close(one, c["out"].reshape(-1, 3072), 4.0, floor=0.5, what="ln_mod single vs shim")


def test_layernorm_modulate_per_row(golden):
    c = golden["layernorm_modulate_per_row"]
    assert torch.equal(ops.layernorm_modulate_shim(c["x"], c["shift"], c["scale"], c["eps"]), c["out"])
    D = c["x"].shape[-1]
    one = ops.norm_scale_shift(c["x"].reshape(-1, D), None, None, c["scale"].reshape(-1, D),
                               c["shift"].reshape(-1, D), "layer", c["eps"])
    assert_bf16_close(one, c["out"].reshape(-1, D), 4.0, floor=0.5, what="per-row ln_mod single vs shim")


def test_gated_residual_bit_exact(golden):
    c = golden["fused_add_gate"]
    out = ops.gated_residual(c["res"], c["x"], c["gate"].unsqueeze(1))
    assert torch.equal(out, c["out"])
    # gate [B, D] per batch item == a per-row [B*L, D] gate on the flattened rows
    c = golden["fused_add_gate_batched"]
    B, L, D = c["res"].shape
    rows_gate = c["gate"][:, None, :].expand(B, L, D).reshape(-1, D)
    out = ops.gated_residual(c["res"].reshape(-1, D), c["x"].reshape(-1, D), rows_gate)
    assert torch.equal(out, c["out"].reshape(-1, D))


def test_rope_tables_bit_exact(golden):
    from joyomni_ops import rope

    for name in ("rope_tables", "rope_tables_t63"):
        c = golden[name]
        pos = rope.grid_positions(c["frames"], c["height"], c["width"], c["t0"])
        cos, sin = rope.rope_3d(pos, c["dims"], c["theta"])
        assert torch.equal(cos, c["cos_full"]) and torch.equal(sin, c["sin_full"]), name
        ch, sh = rope.paired_tables(cos, sin)
        assert torch.equal(ch, c["cos_half"]) and torch.equal(sh, c["sin_half"]), name
        # the oracle's own restatement (the benchmark's CPU arm builds its tables with it)
        (cf, sf), (ch2, sh2) = ops.rope_video_tables(c["frames"], c["height"], c["width"], c["t0"], c["dims"],
                                                     c["theta"])
        assert torch.equal(cf, c["cos_full"]) and torch.equal(sf, c["sin_full"]), name
        assert torch.equal(ch2, c["cos_half"]) and torch.equal(sh2, c["sin_half"]), name


def test_qkv_pack_reference_path(golden):
    """The benchmark's CPU arm for config 1 equals the reference's fallback on the golden case."""
    c = golden["qk_norm_rope_shim"]
    q, k = c["q"], c["k"]
    B, L, H, D = q.shape
    v = torch.randn(B, L, H, D, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    qkv = torch.stack((q, k, v), dim=2).reshape(L, 3 * H * D)
    oq, ok, ov = ops.qkv_pack_reference_path(qkv, H, c["qw"], c["kw"], c["cos"], c["sin"], c["eps"])
    assert torch.equal(oq, c["q_out"][0].transpose(0, 1))
    assert torch.equal(ok, c["k_out"][0].transpose(0, 1))
    assert torch.equal(ov, v[0].transpose(0, 1))


def test_qk_norm_rope(golden):
    c = golden["qk_norm_rope_shim"]
    q, k = c["q"], c["k"]
    B, L, H, D = q.shape
    # shim restatement is bit-exact to the reference's PyTorch path
    qs, ks, kpre = ops.qk_norm_rope_shim(q, k, c["qw"], c["kw"], c["cos"], c["sin"], c["eps"])
    assert torch.equal(qs, c["q_out"]) and torch.equal(ks, c["k_out"]) and torch.equal(kpre, c["k_pre"])
    # kernel semantics (single rounding) vs the shim's norm -> bf16 -> rope: the
    # shim's intermediate bf16 rounding of the O(1) normalised values shows up
    # as up to 2 ulps of O(1) wherever the rotation cancels.
    qo, ko, kp = ops.qk_norm_rope_paired(q.reshape(B, L * H, D), k.reshape(B, L * H, D), L, H, c["eps"],
                                         c["qw"], c["kw"], c["cos"], c["sin"])
    assert torch.equal(kp.view(B, L, H, D), c["k_pre"])  # norm*w rounded once on both sides
    assert_bf16_close(qo.view(B, L, H, D), c["q_out"], 2.0, floor=0.5, what="q single vs shim")
    assert_bf16_close(ko.view(B, L, H, D), c["k_out"], 2.0, floor=0.5, what="k single vs shim")


def test_joint_qkv_pack(golden):
    c = golden["joint_qkv_pack_shim"]
    iq, ik, iv = c["img_qkv"].unbind(2)
    tq, tk, tv = c["txt_qkv"].unbind(2)
    args = (iq, ik, iv, tq, tk, tv, c["cached_k"], c["cached_v"], c["txt_q_weight"], c["txt_k_weight"], c["eps"])
    sq, sk, sv = ops.joint_qkv_pack_shim(*args)
    assert torch.equal(sq, c["out_q"]) and torch.equal(sk, c["out_k"]) and torch.equal(sv, c["out_v"])
    oq, ok, ov = ops.joint_qkv_pack(*args)
    assert torch.equal(ov, c["out_v"])  # V is a pure copy (test_parity_light.py:173)
    n_img, n_cache = iq.shape[1], c["cached_k"].shape[1]
    assert torch.equal(oq[:, :n_img], c["out_q"][:, :n_img])
    assert torch.equal(ok[:, : n_cache + n_img], c["out_k"][:, : n_cache + n_img])
    # text rows: double (kernel/model) vs single (shim) rounding of the norm
    assert_bf16_close(oq, c["out_q"], 1.0, what="joint q")
    assert_bf16_close(ok, c["out_k"], 1.0, what="joint k")


def test_joint_qkv_pack_without_cache(golden):
    c = golden["joint_qkv_pack_nocache"]
    iq, ik, iv = c["img_qkv"].unbind(2)
    tq, tk, tv = c["txt_qkv"].unbind(2)
    args = (iq, ik, iv, tq, tk, tv, None, None, c["txt_q_weight"], c["txt_k_weight"], c["eps"])
    sq, sk, sv = ops.joint_qkv_pack_shim(*args)
    assert torch.equal(sq, c["out_q"]) and torch.equal(sk, c["out_k"]) and torch.equal(sv, c["out_v"])
    oq, ok, ov = ops.joint_qkv_pack(*args)
    assert torch.equal(ov, c["out_v"])
    n_img = iq.shape[1]
    assert torch.equal(oq[:, :n_img], c["out_q"][:, :n_img]) and torch.equal(ok[:, :n_img], c["out_k"][:, :n_img])
    assert_bf16_close(oq, c["out_q"], 1.0, what="joint q, no cache")
    assert_bf16_close(ok, c["out_k"], 1.0, what="joint k, no cache")


def test_cached_kv_rotation(golden):
    c = golden["cached_k_rotation"]
    L = c["cos"].shape[0]
    v0 = torch.zeros_like(c["key0"])
    v1 = torch.zeros_like(c["key1"])
    ok, _ = ops.cached_kv_pack(c["key0"], v0, c["key1"], v1, c["cos"], c["sin"])
    assert ok.shape == c["out"].shape and L == ok.shape[1]
    # same formula, association differs only in x1*c + x0*s vs x0*s + x1*c
    assert_bf16_close(ok, c["out"], 1.0, what="cached rotation")


def test_per_token_quant_bit_exact(golden):
    c = golden["per_token_quant"]
    q, s = ops.per_token_quant_fp8(c["x"])
    assert torch.equal(q.view(torch.uint8), c["q"])
    assert torch.equal(s, c["s"])
    # zero row: the amax clamp gives scale fp32(1e-8) / 448 (not the reference kernel's 0), bytes 0
    assert torch.equal(s[0], torch.tensor([1e-8], dtype=torch.float32) / 448.0)
    assert (q[0].view(torch.uint8) == 0).all()


def test_per_token_quant_edges_bit_exact(golden):
    # negative zeros, amax below the 1e-8 clamp, e4m3 subnormals, |x| near the bf16
    # maximum, one-signed rows, fp16 input
    for name in ("per_token_quant_edges", "per_token_quant_f16"):
        c = golden[name]
        q, s = ops.per_token_quant_fp8(c["x"])
        assert torch.equal(q.view(torch.uint8), c["q"]), name
        assert torch.equal(s, c["s"]), name
    c = golden["per_token_quant_edges"]
    assert (c["q"][0] == 0x80).all()  # -0.0 keeps its sign through the e4m3 cast
    assert (c["q"][1] != 0).any()  # values below the clamp are scaled up, not flushed


def test_weight_quant_bit_exact(golden):
    c = golden["weight_quant"]
    q, s = ops.quantize_weight_per_channel(c["w"])
    assert tuple(q.stride()) == c["q_stride"]
    assert torch.equal(q.contiguous().view(torch.uint8), c["q"])
    assert torch.equal(s, c["s"])
    # per-channel weight quant == per-token quant of the [N, K] weight rows
    qt, st = ops.per_token_quant_fp8(c["w"])
    assert torch.equal(qt.view(torch.uint8), q.t().contiguous().view(torch.uint8))
    assert torch.equal(st.reshape(-1), s.reshape(-1))


def test_gelu_bit_exact(golden):
    c = golden["gelu_tanh"]
    assert torch.equal(ops.gelu_tanh(c["x"]), c["out"])


def test_fp8_gemm_oracle_small():
    # A tiny known-answer: identity-like operands give back the scales.
    a = torch.zeros(4, 16)
    a[torch.arange(4), torch.arange(4)] = 1.0
    b = torch.zeros(16, 3)
    b[0, 0] = 2.0
    b[1, 1] = -4.0
    b[2, 2] = 0.5
    sa = torch.tensor([1.0, 2.0, 0.5, 3.0])
    sb = torch.tensor([1.0, 0.25, 8.0])
    d = ops.fp8_scaled_mm(a.to(ops.FP8), b.to(ops.FP8), sa, sb, None, torch.bfloat16)
    exp = torch.tensor([[2.0, 0, 0], [0, -2.0, 0], [0, 0, 2.0], [0, 0, 0]])
    assert torch.equal(d.float(), exp)


def test_timestep_embedding_known_values():
    t = torch.tensor([0.0, 1.0, 999.0])
    e = ops.timestep_embedding(t, 256)
    assert e.shape == (3, 256)
    # t = 0: cos = 1 (first half after the flip), sin = 0
    assert torch.equal(e[0, :128], torch.ones(128)) and torch.equal(e[0, 128:], torch.zeros(128))
    # frequency 0 is exactly 1: entries are cos(t), sin(t)
    assert abs(e[1, 0].item() - torch.cos(torch.tensor(1.0)).item()) < 1e-7
    assert abs(e[2, 128].item() - torch.sin(torch.tensor(999.0)).item()) < 1e-6


def test_oracle_timestep_mlp_composition():
    """The timestep MLP restatement composes the modules of WanTimeTextImageEmbedding
    (dit.py:574-579, 605-620) in order: Timesteps -> bf16 -> Linear -> SiLU -> Linear ->
    SiLU -> Linear; checked against the same composition with torch.nn modules in fp32
    (bf16 rounding of each materialised tensor is the only difference)."""
    import torch.nn as nn

    g = torch.Generator().manual_seed(0)
    F_, D, P = 64, 96, 192
    l1, l2, l3 = nn.Linear(F_, D), nn.Linear(D, D), nn.Linear(D, P)
    for m in (l1, l2, l3):
        with torch.no_grad():
            m.weight.copy_(torch.randn(m.weight.shape, generator=g) / m.weight.shape[1] ** 0.5)
            m.bias.copy_(0.1 * torch.randn(m.bias.shape, generator=g))
    ws = [t.detach().to(torch.bfloat16) for t in (l1.weight, l1.bias, l2.weight, l2.bias, l3.weight, l3.bias)]
    t = torch.tensor([0.0, 17.5, 999.0])
    vec, s1, s2 = ops.timestep_mlp(t, *ws)
    with torch.no_grad():
        for m, i in ((l1, 0), (l2, 2), (l3, 4)):
            m.weight.copy_(ws[i].float())
            m.bias.copy_(ws[i + 1].float())
        e = ops.timestep_embedding(t, F_).to(torch.bfloat16).float()
        ref = l3(nn.functional.silu(l2(nn.functional.silu(l1(e)))))
    rel = ((vec.float() - ref).norm() / ref.norm()).item()
    assert vec.shape == (3, P) and s1.shape == (3, D) and s2.shape == (3, D)
    assert rel < 2e-2, rel


def test_oracle_gated_residual_gemm_matches_unfused():
    """fp8_scaled_mm_gated_residual = residual + gate * (fp8_scaled_mm in fp32), i.e. the
    unfused chain (GEMM, then torch.addcmul) without the intermediate rounding."""
    g = torch.Generator().manual_seed(1)
    x = torch.randn(33, 64, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(48, 64, generator=g)).to(torch.bfloat16)
    aq, sa = ops.per_token_quant_fp8(x)
    bq, sb = ops.quantize_weight_per_channel(w)
    res = torch.randn(33, 48, generator=g).to(torch.bfloat16)
    gate = (0.1 * torch.randn(1, 48, generator=g)).to(torch.bfloat16)
    fused = ops.fp8_scaled_mm_gated_residual(aq, bq, sa, sb, None, res, gate)
    prod = ops.fp8_scaled_mm(aq, bq, sa, sb, None, torch.float32)
    assert torch.equal(fused, (res.float() + gate.float() * prod).to(torch.bfloat16))
    unfused = ops.gated_residual(res, prod.to(torch.bfloat16), gate)
    assert (fused.float() - unfused.float()).abs().max().item() <= 2 * 2.0 ** -7 * res.float().abs().max().item()
