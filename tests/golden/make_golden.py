"""Generate tests/golden/reference_golden.pt by running the REFERENCE's own Python.

Run once in a container that has the reference checkout (it is not needed on
the GPU box; only the resulting .pt travels):

    python tests/golden/make_golden.py [REFERENCE_ROOT]

REFERENCE_ROOT defaults to the JOYOMNI_REFERENCE environment variable.  The
reference modules are imported by file path:

* deploy/xvideo/models/dit/sgl_fused_ops.py  (the call-site shim; its PyTorch
  path runs because no native joyomni_ops is importable here),
* deploy/xvideo/models/dit/fp8_linear.py     (per-token / per-channel FP8 quant),
* deploy/xvideo/models/dit/rope.py           (RoPE tables and rotation),

and torch.nn.functional.gelu(approximate="tanh"), which is the reference's own
call at deploy/xvideo/models/dit/dit.py:87-89.  Every case is seeded; inputs and
the reference outputs are stored side by side.
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import torch


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root: Path) -> None:
    # The shim must not find a native joyomni_ops (ours or the reference's).
    sys.path = [p for p in sys.path if "joyai-video-edit_b200" not in p]
    dit = ref_root / "deploy" / "xvideo" / "models" / "dit"
    sgl = _load("ref_sgl_fused_ops", dit / "sgl_fused_ops.py")
    fp8 = _load("ref_fp8_linear", dit / "fp8_linear.py")
    rope = _load("ref_rope", dit / "rope.py")
    assert sgl.available() is False, "reference shim must take its PyTorch path"
    assert fp8.available() is False

    bf = torch.bfloat16
    cases = {}

    def gen(seed):
        return torch.Generator().manual_seed(seed)

    # --- rmsnorm (_torch_rmsnorm, rmsnorm_qk_bf16 fallback) ---------------------
    for i, (M, N) in enumerate([(7, 3072), (5, 136), (3, 4096)]):
        g = gen(100 + i)
        x = torch.randn(M, N, generator=g).to(bf)
        w = (1 + 0.02 * torch.randn(N, generator=g)).to(bf)
        cases[f"rmsnorm_{M}x{N}"] = dict(x=x, w=w, eps=1e-6, out=sgl._torch_rmsnorm(x, w, 1e-6))
    g = gen(110)
    x = torch.randn(2, 3, 4, 128, generator=g).to(bf)
    w = (1 + 0.02 * torch.randn(128, generator=g)).to(bf)
    cases["rmsnorm_qk_bf16"] = dict(x=x, w=w, eps=1e-6, out=sgl.rmsnorm_qk_bf16(x, w, 1e-6))

    # --- LayerNorm + modulate (shim PyTorch path) -------------------------------
    g = gen(200)
    x = torch.randn(1, 9, 3072, generator=g).to(bf)
    shift = (0.1 * torch.randn(1, 3072, generator=g)).to(bf)
    scale = (0.1 * torch.randn(1, 3072, generator=g)).to(bf)
    cases["layernorm_modulate"] = dict(
        x=x, shift=shift, scale=scale, eps=1e-6,
        out=sgl.fused_layernorm_modulate(x, shift=shift, scale=scale, eps=1e-6))

    # --- gated residual ----------------------------------------------------------
    g = gen(300)
    res = torch.randn(1, 9, 3072, generator=g).to(bf)
    xx = torch.randn(1, 9, 3072, generator=g).to(bf)
    gate = (0.1 * torch.randn(1, 3072, generator=g)).to(bf)
    cases["fused_add_gate"] = dict(res=res, x=xx, gate=gate, out=sgl.fused_add_gate(res, xx, gate))

    # --- RoPE tables (rope.get_1d_rotary_pos_embed + prepare_fused_rope) --------
    F_, H_, W_, t0 = 2, 3, 4, 5
    t = (torch.arange(F_).float() + t0).repeat_interleave(H_ * W_)
    h = torch.arange(H_).float().repeat_interleave(W_).repeat(F_)
    w_ = torch.arange(W_).float().repeat(F_ * H_)
    cos_l, sin_l = [], []
    for dim, pos in zip((44, 42, 42), (t, h, w_)):
        c, s = rope.get_1d_rotary_pos_embed(dim, pos, theta=10000.0)
        cos_l.append(c)
        sin_l.append(s)
    cos_full, sin_full = torch.cat(cos_l, 1), torch.cat(sin_l, 1)
    cos_h, sin_h = sgl.prepare_fused_rope((cos_full, sin_full), head_dim=128, device=torch.device("cpu"))
    cases["rope_tables"] = dict(frames=F_, height=H_, width=W_, t0=t0, dims=(44, 42, 42), theta=10000.0,
                                cos_full=cos_full, sin_full=sin_full, cos_half=cos_h, sin_half=sin_h)

    # --- q/k norm + rope (shim PyTorch path) -------------------------------------
    g = gen(400)
    L, Hh = F_ * H_ * W_, 4
    q = torch.randn(1, L, Hh, 128, generator=g).to(bf)
    k = torch.randn(1, L, Hh, 128, generator=g).to(bf)
    qw = (1 + 0.02 * torch.randn(128, generator=g)).to(bf)
    kw = (1 + 0.02 * torch.randn(128, generator=g)).to(bf)
    qo, ko, kpre = sgl.fused_qk_norm_rope_3d(q, k, qw, kw, (cos_h, sin_h), eps=1e-6, return_k_pre_rope=True)
    cases["qk_norm_rope_shim"] = dict(q=q, k=k, qw=qw, kw=kw, cos=cos_h, sin=sin_h, eps=1e-6,
                                      q_out=qo, k_out=ko, k_pre=kpre)

    # --- joint pack (shim PyTorch path; V strided like the model's unbind view) --
    g = gen(500)
    img_qkv = torch.randn(1, 17, 3, 4, 128, generator=g).to(bf)
    txt_qkv = torch.randn(1, 11, 3, 4, 128, generator=g).to(bf)
    ck = torch.randn(1, 9, 4, 128, generator=g).to(bf)
    cv = torch.randn(1, 9, 4, 128, generator=g).to(bf)
    tqw = torch.randn(128, generator=g).to(bf)
    tkw = torch.randn(128, generator=g).to(bf)
    iq, ik, iv = img_qkv.unbind(2)
    tq, tk, tv = txt_qkv.unbind(2)
    oq, ok, ov = sgl.fused_joint_qkv_pack(iq, ik, iv, tq, tk, tv, ck, cv, tqw, tkw, 1e-6)
    cases["joint_qkv_pack_shim"] = dict(img_qkv=img_qkv, txt_qkv=txt_qkv, cached_k=ck, cached_v=cv,
                                        txt_q_weight=tqw, txt_k_weight=tkw, eps=1e-6,
                                        out_q=oq, out_k=ok, out_v=ov)

    # --- cached K rotation (rope.apply_rotary_emb, the non-fused cache path) -----
    g = gen(600)
    k0 = torch.randn(1, 13, 4, 128, generator=g).to(bf)
    k1 = torch.randn(1, 7, 4, 128, generator=g).to(bf)
    cpair = torch.randn(20, 64, generator=g)
    spair = torch.randn(20, 64, generator=g)
    cfull = cpair.repeat_interleave(2, dim=-1).contiguous()
    sfull = spair.repeat_interleave(2, dim=-1).contiguous()
    rot = rope.apply_rotary_emb(torch.cat((k0, k1), 1), (cfull, sfull))
    cases["cached_k_rotation"] = dict(key0=k0, key1=k1, cos=cfull, sin=sfull, out=rot)

    # --- FP8 per-token / per-channel quant ---------------------------------------
    g = gen(700)
    x = torch.randn(67, 4096, generator=g).to(bf)
    x[0].zero_()  # test_parity_light.py:117-119
    x[1] *= 1e-3
    x[2] *= 300.0
    qq, ss = fp8._quantize_per_token_impl(x)
    cases["per_token_quant"] = dict(x=x, q=qq.view(torch.uint8), s=ss)
    g = gen(701)
    wt = (0.02 * torch.randn(48, 3072, generator=g)).to(bf)
    wq, ws = fp8._quantize_weight_per_channel(wt)
    cases["weight_quant"] = dict(w=wt, q=wq.contiguous().view(torch.uint8), q_stride=tuple(wq.stride()), s=ws)

    # --- edge cases of the same reference functions -------------------------------
    # fp16 and fp32 inputs of _torch_rmsnorm (the native op takes fp32/fp16/bf16)
    for i, dt in enumerate((torch.float16, torch.float32)):
        g = gen(120 + i)
        x = torch.randn(6, 1000, generator=g).to(dt)
        w = (1 + 0.02 * torch.randn(1000, generator=g)).to(dt)
        cases[f"rmsnorm_{str(dt).split('.')[-1]}"] = dict(x=x, w=w, eps=1e-6, out=sgl._torch_rmsnorm(x, w, 1e-6))
    # per-row modulation through the call site's non-native path
    g = gen(210)
    x = torch.randn(1, 5, 1024, generator=g).to(bf)
    shift = (0.1 * torch.randn(1, 5, 1024, generator=g)).to(bf)
    scale = (0.1 * torch.randn(1, 5, 1024, generator=g)).to(bf)
    cases["layernorm_modulate_per_row"] = dict(
        x=x, shift=shift, scale=scale, eps=1e-6,
        out=sgl.fused_layernorm_modulate(x, shift=shift, scale=scale, eps=1e-6))
    # per-batch gate (gate [B, D] broadcast over each item's tokens)
    g = gen(310)
    res = torch.randn(2, 3, 512, generator=g).to(bf)
    xx = torch.randn(2, 3, 512, generator=g).to(bf)
    gate = (0.1 * torch.randn(2, 512, generator=g)).to(bf)
    cases["fused_add_gate_batched"] = dict(res=res, x=xx, gate=gate, out=sgl.fused_add_gate(res, xx, gate))
    # RoPE tables at the largest start frame the streaming loop uses (t0 = 63)
    F2, H2, W2, t02 = 1, 5, 7, 63
    t = (torch.arange(F2).float() + t02).repeat_interleave(H2 * W2)
    h = torch.arange(H2).float().repeat_interleave(W2).repeat(F2)
    w_ = torch.arange(W2).float().repeat(F2 * H2)
    cos_l, sin_l = [], []
    for dim, pos in zip((44, 42, 42), (t, h, w_)):
        c, s = rope.get_1d_rotary_pos_embed(dim, pos, theta=10000.0)
        cos_l.append(c)
        sin_l.append(s)
    cf2, sf2 = torch.cat(cos_l, 1), torch.cat(sin_l, 1)
    ch2, sh2 = sgl.prepare_fused_rope((cf2, sf2), head_dim=128, device=torch.device("cpu"))
    cases["rope_tables_t63"] = dict(frames=F2, height=H2, width=W2, t0=t02, dims=(44, 42, 42), theta=10000.0,
                                    cos_full=cf2, sin_full=sf2, cos_half=ch2, sin_half=sh2)
    # joint pack without a cache (the first chunk of a stream)
    g = gen(510)
    img_qkv = torch.randn(1, 6, 3, 2, 128, generator=g).to(bf)
    txt_qkv = torch.randn(1, 4, 3, 2, 128, generator=g).to(bf)
    tqw = torch.randn(128, generator=g).to(bf)
    tkw = torch.randn(128, generator=g).to(bf)
    iq, ik, iv = img_qkv.unbind(2)
    tq, tk, tv = txt_qkv.unbind(2)
    oq, ok, ov = sgl.fused_joint_qkv_pack(iq, ik, iv, tq, tk, tv, None, None, tqw, tkw, 1e-6)
    cases["joint_qkv_pack_nocache"] = dict(img_qkv=img_qkv, txt_qkv=txt_qkv, txt_q_weight=tqw, txt_k_weight=tkw,
                                           eps=1e-6, out_q=oq, out_k=ok, out_v=ov)
    # per-token quant: fp16 input, negative zeros, an all-tiny row (amax below the
    # 1e-8 clamp), one dominant element (the rest in e4m3's subnormal range),
    # values near the bf16 maximum, and one-signed rows
    g = gen(710)
    x = torch.randn(9, 256, generator=g)
    x[0] = -0.0
    x[1] *= 1e-10
    x[2] *= 1e-3
    x[2, 17] = 50.0
    x[3] *= 1e36
    x[4] = x[4].abs()
    x[5] = -x[5].abs()
    x[6, ::2] = 0.0
    xb = x.to(bf)
    qq, ss = fp8._quantize_per_token_impl(xb)
    cases["per_token_quant_edges"] = dict(x=xb, q=qq.view(torch.uint8), s=ss)
    xh = torch.randn(17, 512, generator=gen(711)).to(torch.float16)
    xh[0] *= 2000.0  # |x| up to ~1e4, inside fp16's range
    xh[1] = 0.0
    qq, ss = fp8._quantize_per_token_impl(xh)
    cases["per_token_quant_f16"] = dict(x=xh, q=qq.view(torch.uint8), s=ss)

    # --- GELU-tanh (the reference's own call) ------------------------------------
    g = gen(800)
    x = (torch.randn(6, 1024, generator=g) * torch.tensor([0.1, 1.0, 3.0, 6.0, 10.0, 30.0])[:, None]).to(bf)
    cases["gelu_tanh"] = dict(x=x, out=torch.nn.functional.gelu(x, approximate="tanh"))

    # store compact copies (a saved view would carry its whole base storage)
    cases = {n: {k: (v.clone().contiguous() if torch.is_tensor(v) else v) for k, v in c.items()}
             for n, c in cases.items()}
    out = Path(__file__).resolve().parent / "reference_golden.pt"
    torch.save(dict(cases=cases, generator="tests/golden/make_golden.py", torch=torch.__version__), out)
    print(f"wrote {out} ({out.stat().st_size} bytes, {len(cases)} cases)")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("JOYOMNI_REFERENCE")
    if not root:
        raise SystemExit("usage: make_golden.py REFERENCE_ROOT (or set JOYOMNI_REFERENCE)")
    main(Path(root))
