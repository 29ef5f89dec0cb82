"""CPU oracle functions (torch, fp32 math).  Test infrastructure only.

Conventions: inputs are CPU tensors; outputs are rounded to the output dtype
exactly once unless the cited reference rounds more often (stated per function).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0  # torch.finfo(torch.float8_e4m3fn).max


# ----------------------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """y = dtype((x * rsqrt(mean(x^2) + eps)) * w), fp32 math, one rounding.

    deploy/xvideo/models/dit/sgl_fused_ops.py:202-209 (_torch_rmsnorm); the
    reference kernel computes the same formula (joyomni_ops/csrc/rmsnorm.cu:60-84).
    """
    xf = x.float()
    out = xf * torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + eps)
    return (out * w.float()).to(x.dtype)


def rmsnorm_model(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """The model's RMSNorm module: normalise -> dtype, then * weight -> dtype (two roundings).

    deploy/xvideo/models/dit/dit.py:289-296.
    """
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return n * w.to(x.dtype)


def norm_scale_shift(x, gamma, beta, scale, shift, norm_type: str, eps: float) -> torch.Tensor:
    """Norm(x; gamma, beta) * (1 + scale) + shift in fp32, one rounding.

    LayerNorm: joyomni_ops/tests/test_parity_light.py:51-56 and the kernel formula
    joyomni_ops/csrc/fused_norm_scale_shift.cu:296-307; RMS: the same kernel's
    rms branch (x * rstd * g) * (1 + scale) + shift.  scale/shift are [M, N] or
    broadcast [1, N]; gamma/beta may be None.
    """
    xf = x.float()
    if norm_type == "layer":
        mean = xf.mean(-1, keepdim=True)
        var = (xf - mean).pow(2).mean(-1, keepdim=True)
        n = (xf - mean) * torch.rsqrt(var + eps)
        if gamma is not None:
            n = n * gamma.float()
        if beta is not None:
            n = n + beta.float()
    elif norm_type == "rms":
        n = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        if gamma is not None:
            n = n * gamma.float()
    else:
        raise ValueError(norm_type)
    return (n * (1 + scale.float()) + shift.float()).to(x.dtype)


def layernorm_modulate_shim(x, shift, scale, eps: float) -> torch.Tensor:
    """The call site's non-native path: F.layer_norm -> dtype, then dtype arithmetic.

    deploy/xvideo/models/dit/sgl_fused_ops.py:90-91 (rounds after each op).
    """
    D = x.shape[-1]
    out = F.layer_norm(x, (D,), eps=eps)
    return out * (1 + scale) + shift


# ----------------------------------------------------------------------------- residual / activations
def gated_residual(res, x, gate) -> torch.Tensor:
    """torch.addcmul(residual, x, gate): deploy/xvideo/models/dit/sgl_fused_ops.py:302-305.

    gate is [N], [1, N] or [M, N] (broadcast over rows).
    """
    return torch.addcmul(res, x, gate.reshape(-1, res.shape[-1]) if gate.dim() > 1 else gate)


def gated_residual_norm_scale_shift(res, x, gate, scale, shift, norm_type, eps, gamma=None, beta=None):
    """h = addcmul(res, x, gate) (rounded), then norm_scale_shift(h): dit.py:525-534."""
    h = gated_residual(res, x, gate)
    return h, norm_scale_shift(h, gamma, beta, scale, shift, norm_type, eps)


def gelu_tanh(x) -> torch.Tensor:
    """F.gelu(x, approximate="tanh") on the CPU: deploy/xvideo/models/dit/dit.py:87-89."""
    return F.gelu(x, approximate="tanh")


def silu_mul(a, b) -> torch.Tensor:
    """dtype(silu(a) * b) in fp32 (SiLU-gated MLP; no reference op -- parity unpinned)."""
    return (F.silu(a.float()) * b.float()).to(a.dtype)


def timestep_embedding(t, dim=256, flip_sin_to_cos=True, downscale_freq_shift=0.0, scale=1.0,
                       max_period=10000.0) -> torch.Tensor:
    """Sinusoidal timestep projection, fp32 [B, dim].

    Restates the published diffusers 0.36.0 ``get_timestep_embedding`` used by
    ``Timesteps(256, flip_sin_to_cos=True, downscale_freq_shift=0)`` at
    deploy/xvideo/models/dit/dit.py:574-575,614.  diffusers is a third-party
    dependency absent from the reference tree (pinned at requirements.txt:8):
    parity unpinned.
    """
    half = dim // 2
    exponent = -math.log(max_period) * torch.arange(0, half, dtype=torch.float32)
    exponent = exponent / (half - downscale_freq_shift)
    emb = torch.exp(exponent)
    emb = t[:, None].float() * emb[None, :]
    emb = scale * emb
    emb = torch.cat([torch.sin(emb), torch.cos(emb)], dim=-1)
    if flip_sin_to_cos:
        emb = torch.cat([emb[:, half:], emb[:, :half]], dim=-1)
    if dim % 2 == 1:
        emb = F.pad(emb, (0, 1, 0, 0))
    return emb


def fp8_scaled_mm_gated_residual(a_q, b_q, scale_a, scale_b, bias, residual, gate) -> torch.Tensor:
    """residual + gate * (the fp8_scaled_mm result before its rounding): the down
    projection and torch.addcmul(res, x, gate) (dit.py:536-538, sgl_fused_ops.py:302-305)
    with the product kept in fp32, one rounding to the residual's dtype."""
    acc = (a_q.double() @ b_q.double()).float()
    d = (acc * scale_b.reshape(1, -1).float()) * scale_a.reshape(-1, 1).float()
    if bias is not None:
        d = d + bias.float().reshape(1, -1)
    return (residual.float() + gate.float().reshape(1, -1) * d).to(residual.dtype)


def linear_bf16(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor]) -> torch.Tensor:
    """bf16 nn.Linear as the GPU reference runs it (cuBLAS): fp32 accumulation, bias
    added in fp32, one rounding to bf16."""
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return y.to(torch.bfloat16)


def silu_bf16(x: torch.Tensor) -> torch.Tensor:
    """nn.SiLU on a bf16 tensor: fp32 math on the bf16 values, rounded to bf16."""
    return F.silu(x.float()).to(torch.bfloat16)


def timestep_mlp(t, w1, b1, w2, b2, w3, b3, max_period=10000.0):
    """WanTimeTextImageEmbedding timestep branch (deploy/xvideo/models/dit/dit.py:574-579,
    605-620): Timesteps(freq, flip_sin_to_cos=True, shift=0) -> bf16 -> time_embedder
    (linear_1, SiLU, linear_2) -> act_fn SiLU -> time_proj.  Returns (vec, s1, s2) with
    s1 = silu(linear_1(e)) and s2 = silu(temb), the two tensors the modules materialise
    between the Linears."""
    e = timestep_embedding(t, w1.shape[1], True, 0.0, 1.0, max_period).to(torch.bfloat16)
    s1 = silu_bf16(linear_bf16(e, w1, b1))
    s2 = silu_bf16(linear_bf16(s1, w2, b2))
    return linear_bf16(s2, w3, b3), s1, s2


# ----------------------------------------------------------------------------- q/k norm + rope
def _rope_pairs(xn: torch.Tensor, c: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    x1, x2 = xn[..., 0::2], xn[..., 1::2]
    o = torch.empty_like(xn)
    o[..., 0::2] = x1 * c - x2 * s
    o[..., 1::2] = x1 * s + x2 * c
    return o


def qk_norm_rope_paired(q, k, seq_len, num_heads, eps, qw, kw, cos, sin):
    """(q_out, k_out, k_pre_rope) of fused_qk_norm_rope_3d_paired, single rounding.

    joyomni_ops/tests/test_parity_light.py:93-110 (the fp32 reference of the
    kernel joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:141-232).
    q, k: [B, L*H, D]; cos, sin: [L, D/2].
    """
    B, M, D = q.shape
    c = cos.float().view(seq_len, 1, D // 2)
    s = sin.float().view(seq_len, 1, D // 2)

    def one(x, w):
        xf = x.float().view(B, seq_len, num_heads, D)
        xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
        return xn, _rope_pairs(xn, c, s).view(B, M, D).to(torch.bfloat16)

    _, qo = one(q, qw)
    kn, ko = one(k, kw)
    return qo, ko, kn.view(B, M, D).to(torch.bfloat16)


def qk_norm_rope_shim(q, k, qw, kw, cos, sin, eps):
    """The call site's non-native path (sgl_fused_ops.py:170-199): _torch_rmsnorm -> bf16,
    then full-width RoPE in fp32 -> bf16.  q, k: [B, L, H, D]; cos, sin: [L, D/2]."""
    B, L, H, D = q.shape
    qn = rmsnorm(q, qw, eps)
    kn = rmsnorm(k, kw, eps)
    cf = cos.repeat_interleave(2, dim=-1).reshape(1, L, 1, D).float()
    sf = sin.repeat_interleave(2, dim=-1).reshape(1, L, 1, D).float()

    def apply(x):
        xf = x.float()
        pairs = xf.reshape(*x.shape[:-1], -1, 2)
        rot = torch.stack((-pairs[..., 1], pairs[..., 0]), dim=-1).flatten(-2)
        return (xf * cf + rot * sf).to(x.dtype)

    return apply(qn), apply(kn), kn


def rope_video_tables(frames: int, height: int, width: int, t0: int, dims=(44, 42, 42), theta: float = 10000.0):
    """(cos_full, sin_full) fp32 [F*H*W, sum(dims)] and (cos_half, sin_half) bf16 [F*H*W, sum(dims)/2]
    for a frame-major (t, h, w) token grid whose frames start at t0.

    Per axis get_1d_rotary_pos_embed (deploy/xvideo/models/dit/rope.py:31-52: freqs =
    1/theta^(arange(0, d, 2)/d), outer product with the positions, cos/sin repeat-interleaved),
    concatenated over (t, h, w) as get_rotary_pos_embed_from_ids does (dit.py:896-934), then
    prepare_fused_rope's every-other-column bf16 tables (sgl_fused_ops.py:94-119).
    """
    t = (torch.arange(frames, dtype=torch.float32) + float(t0)).repeat_interleave(height * width)
    h = torch.arange(height, dtype=torch.float32).repeat_interleave(width).repeat(frames)
    w = torch.arange(width, dtype=torch.float32).repeat(frames * height)
    cos_l, sin_l = [], []
    for d, pos in zip(dims, (t, h, w)):
        freqs = 1.0 / (theta ** (torch.arange(0, d, 2)[: d // 2].float() / d))
        ang = torch.outer(pos, freqs)
        cos_l.append(ang.cos().repeat_interleave(2, dim=1))
        sin_l.append(ang.sin().repeat_interleave(2, dim=1))
    cos, sin = torch.cat(cos_l, 1), torch.cat(sin_l, 1)
    return (cos, sin), (cos[:, ::2].to(torch.bfloat16).contiguous(), sin[:, ::2].to(torch.bfloat16).contiguous())


def qkv_pack_reference_path(qkv, num_heads, qw, kw, cos, sin, eps):
    """Config 1 as the reference computes it without its native ops, step for step.

    The rearrange "B L (K H D) -> K B L H D" of the QKV projection (dit.py:409-411, strided
    views), the fused_qk_norm_rope_3d fallback (sgl_fused_ops.py:170-199: _torch_rmsnorm of
    the strided q and k -> bf16, then the full-width rotation in fp32 -> bf16; restated by
    qk_norm_rope_shim, which the golden vectors pin bit-exactly), and q/k/v materialised
    head-major [H, L, D] as config 1 asks.  The timed CPU arm of the benchmark.
    """
    L = qkv.shape[0]
    D = qkv.shape[1] // (3 * num_heads)
    x = qkv.view(1, L, 3, num_heads, D)
    q, k, v = x.unbind(2)
    qo, ko, _ = qk_norm_rope_shim(q, k, qw, kw, cos, sin, eps)
    return tuple(t[0].transpose(0, 1).contiguous() for t in (qo, ko, v))


def qkv_norm_rope_pack(qkv, num_heads, qw, kw, cos, sin, eps, head_major=True, with_pre=False):
    """q, k, v (and k_pre_rope) from the QKV projection output in one pass.

    Composition of dit.py:409-411 (rearrange "L (K H D) -> K L H D"),
    qk_norm_rope_paired above (single rounding), and a transpose to head-major
    [H, L, D] (or token-major [L, H, D]).
    """
    L = qkv.shape[0]
    D = qkv.shape[1] // (3 * num_heads)
    x = qkv.view(L, 3, num_heads, D)
    q = x[:, 0].reshape(1, L * num_heads, D)
    k = x[:, 1].reshape(1, L * num_heads, D)
    qo, ko, kpre = qk_norm_rope_paired(q, k, L, num_heads, eps, qw, kw, cos, sin)
    outs = [qo.view(L, num_heads, D), ko.view(L, num_heads, D), x[:, 2].clone(), kpre.view(L, num_heads, D)]
    if head_major:
        outs = [o.transpose(0, 1).contiguous() for o in outs]
    return tuple(outs) if with_pre else tuple(outs[:3])


def joint_qkv_pack(img_q, img_k, img_v, txt_q, txt_k, txt_v, cached_k, cached_v, qw, kw, eps):
    """[img|norm(txt)], [cache|img|norm(txt)], [cache|img|txt] with the text RMSNorm
    rounded twice (normalised -> bf16, then * w -> bf16).

    joyomni_ops/tests/test_parity_light.py:160-169, which the reference kernel
    (joyomni_ops/csrc/fused_joint_qkv_pack.cu:59-79) matches.
    """

    def norm(x, w):
        xf = x.float()
        n = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)).to(torch.bfloat16)
        return n * w

    q = torch.cat((img_q, norm(txt_q, qw)), dim=1)
    ks = ([cached_k] if cached_k is not None else []) + [img_k, norm(txt_k, kw)]
    vs = ([cached_v] if cached_v is not None else []) + [img_v, txt_v]
    return q.contiguous(), torch.cat(ks, dim=1).contiguous(), torch.cat(vs, dim=1).contiguous()


def joint_qkv_pack_shim(img_q, img_k, img_v, txt_q, txt_k, txt_v, cached_k, cached_v, qw, kw, eps):
    """The call site's non-native path (sgl_fused_ops.py:257-265): single-rounding text norm."""
    tq = rmsnorm(txt_q, qw, eps).to(txt_v.dtype)
    tk = rmsnorm(txt_k, kw, eps).to(txt_v.dtype)
    q = torch.cat((img_q, tq), dim=1)
    k = torch.cat((img_k, tk), dim=1)
    v = torch.cat((img_v, txt_v), dim=1)
    if cached_k is not None:
        k = torch.cat((cached_k, k), dim=1)
        v = torch.cat((cached_v, v), dim=1)
    return q, k, v


def cached_kv_pack(key0, value0, key1, value1, cos, sin):
    """Concatenate pre-RoPE K/V segments and rotate K with fp32 full-width tables.

    joyomni_ops/tests/test_parity_light.py:189-196; the pair (2m, 2m+1) uses
    table entry 2m for both members, as the kernel does
    (joyomni_ops/csrc/fused_joint_qkv_pack.cu:209-216) -- identical to the test
    for the repeat-interleaved tables the model builds (rope.py:49-50).
    """
    ks = [key0] + ([key1] if key1 is not None else [])
    vs = [value0] + ([value1] if value1 is not None else [])
    src = torch.cat(ks, dim=1).float()
    B, L, H, D = src.shape
    c = cos.view(L, D)[:, 0::2].reshape(1, L, 1, D // 2)
    s = sin.view(L, D)[:, 0::2].reshape(1, L, 1, D // 2)
    return _rope_pairs(src, c, s).to(torch.bfloat16), torch.cat(vs, dim=1).contiguous()


# ----------------------------------------------------------------------------- FP8
def per_token_quant_fp8(x) -> Tuple[torch.Tensor, torch.Tensor]:
    """(q e4m3 [M, N], scale fp32 [M, 1]): deploy/xvideo/models/dit/fp8_linear.py:38-43."""
    absmax = x.abs().amax(dim=1, keepdim=True).float().clamp_min(1e-8)
    scale = absmax / FP8_MAX
    q = (x.float() / scale).clamp(-FP8_MAX, FP8_MAX).to(FP8)
    return q, scale


def quantize_weight_per_channel(w) -> Tuple[torch.Tensor, torch.Tensor]:
    """(w_q e4m3 [K, N] column-major, scale fp32 [1, N]) of a Linear weight [N, K].

    deploy/xvideo/models/dit/fp8_linear.py:77-85.
    """
    w_kn = w.t().contiguous()
    K, N = w_kn.shape
    absmax = w_kn.abs().amax(dim=0).to(torch.float32).clamp_min(1e-8)
    scale = absmax / FP8_MAX
    w_q_rm = (w_kn.float() / scale.unsqueeze(0)).clamp(-FP8_MAX, FP8_MAX).to(FP8)
    return w_q_rm.t().contiguous().t(), scale.reshape(1, N).contiguous()


def rmsnorm_quant_fp8(x, w, eps):
    """per_token_quant_fp8(_torch_rmsnorm(x, w, eps)): the unfused reference chain."""
    return per_token_quant_fp8(rmsnorm(x, w, eps))


def norm_scale_shift_quant_fp8(x, gamma, beta, scale, shift, norm_type, eps):
    """per_token_quant_fp8(norm_scale_shift(...)): dit.py:402-408 -> fp8_linear.py:133-140."""
    return per_token_quant_fp8(norm_scale_shift(x, gamma, beta, scale, shift, norm_type, eps))


def fp8_scaled_mm(a_q, b_q, scale_a, scale_b, bias: Optional[torch.Tensor], out_dtype) -> torch.Tensor:
    """D = out_dtype(scale_a * (A @ B * scale_b) (+ bias)), the epilogue order of the
    reference sm100 kernel's EVT (joyomni_ops/csrc/fp8_gemm.cu:834-861): acc * sB,
    then * sA (+ bias), fp32, one rounding.  The dot products are taken in float64
    (exact e4m3 products, near-exact sums) -- a restatement, parity unpinned.
    """
    acc = (a_q.double() @ b_q.double()).float()
    t = acc * scale_b.reshape(1, -1).float()
    d = t * scale_a.reshape(-1, 1).float()
    if bias is not None:
        d = d + bias.float().reshape(1, -1)
    return d.to(out_dtype)


def qkv_text_pack(qkv, num_heads, qw, kw, eps):
    """Text rows of the joint pack: q/k RMSNorm with the model's double rounding
    (joyomni_ops/tests/test_parity_light.py:160-165), no RoPE; v copied.
    qkv [L, 3*H*D] -> token-major q, k, v [L, H, D]."""
    L = qkv.shape[0]
    D = qkv.shape[1] // (3 * num_heads)
    x = qkv.view(L, 3, num_heads, D)

    def norm(t, w):
        tf = t.float()
        n = (tf * torch.rsqrt(tf.square().mean(-1, keepdim=True) + eps)).to(torch.bfloat16)
        return n * w

    return norm(x[:, 0], qw), norm(x[:, 1], kw), x[:, 2].clone()


def attention(q, k, v):
    """Non-causal softmax attention in fp32 on token-major [S, H, D] tensors -> dtype [Sq, H*D]
    (the math of dit.py:154-168 / torch SDPA)."""
    qf, kf, vf = q.float().transpose(0, 1), k.float().transpose(0, 1), v.float().transpose(0, 1)
    s = (qf @ kf.transpose(1, 2)) / math.sqrt(q.shape[-1])
    o = torch.softmax(s, dim=-1) @ vf
    return o.transpose(0, 1).reshape(q.shape[0], -1).to(q.dtype)


def fp8_linear(xq, xs, w):
    """Fp8Linear.forward on already-quantised input (fp8_linear.py:139-141); w has wq, ws, bias."""
    return fp8_scaled_mm(xq, w.wq, xs, w.ws, w.bias, torch.bfloat16)


def block_stream_out(x, attn, w, m, eps=1e-6):
    """Second half of one stream of MMDoubleStreamBlock.forward (dit.py:525-538), FP8 path."""
    gate1, shift2, scale2, gate2 = m[2], m[3], m[4], m[5]
    aq, asc = per_token_quant_fp8(attn)
    proj = fp8_linear(aq, asc, w.proj)
    h, y = gated_residual_norm_scale_shift(x, proj, gate1, scale2, shift2, "layer", eps)
    hq, hs = per_token_quant_fp8(y)
    up = fp8_linear(hq, hs, w.up)
    gq, gs = per_token_quant_fp8(gelu_tanh(up))
    down = fp8_linear(gq, gs, w.down)
    return gated_residual(h, down, gate2)


def block_forward(img, txt, vec, cos, sin, w, cache_k, cache_v, heads, eps=1e-6):
    """MMDoubleStreamBlock.forward for one chunk (dit.py:360-558), FP8 path, composed of the
    oracle ops above; cache_k/v: token-major [cache_len, H, D] (post-RoPE)."""
    def mod(table):
        m = (table + vec)
        return [m[i:i + 1] for i in range(6)]

    mi, mt = mod(w.img.mod_table), mod(w.txt.mod_table)
    outs = []
    for x, ws, m, rope in ((img, w.img, mi, True), (txt, w.txt, mt, False)):
        xq, xs = norm_scale_shift_quant_fp8(x, None, None, m[1], m[0], "layer", eps)
        qkv = fp8_linear(xq, xs, ws.qkv)
        if rope:
            outs.append(qkv_norm_rope_pack(qkv, heads, ws.q_norm, ws.k_norm, cos, sin, eps, head_major=False))
        else:
            outs.append(qkv_text_pack(qkv, heads, ws.q_norm, ws.k_norm, eps))
    (qi, ki, vi), (qt, kt, vt) = outs
    attn = attention(torch.cat([qi, qt]), torch.cat([cache_k, ki, kt]), torch.cat([cache_v, vi, vt]))
    L = img.shape[0]
    return block_stream_out(img, attn[:L], w.img, mi, eps), block_stream_out(txt, attn[L:], w.txt, mt, eps)


# ----------------------------------------------------------------------------- helpers
def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |x| (1 ulp of the value), as fp32."""
    xf = x.float().abs()
    e = torch.floor(torch.log2(xf.clamp_min(2.0 ** -126)))
    return torch.pow(2.0, e - 7)


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of the bf16 ulp of b (elementwise, fp32)."""
    return (a.float() - b.float()).abs() / bf16_ulp(b)
