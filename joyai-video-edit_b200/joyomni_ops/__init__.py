"""joyomni_ops -- B200-native (sm_100a) drop-in for JoyAI-Video-Edit's op library.

Same import name, same ``torch.ops.joyomni_ops`` schemas, same Python wrappers
and FakeTensor registrations as the reference package
(joyomni_ops/joyomni_ops/__init__.py:1-153, schemas joyomni_ops/csrc/pybind.cpp:52-75),
so ``deploy/xvideo/models/dit/sgl_fused_ops.py`` and ``fp8_linear.py`` bind to it
unchanged.  Every op is a hand-written sm_100a CUDA kernel in
``libjoyomni_b200.so`` reached through its C ABI (``include/joyomni_b200.h``);
``_C.so`` only registers the torch ops.  There is no CPU or eager fallback: the
ops are registered for the CUDA dispatch key only, and importing without the
built extension raises ImportError exactly like the reference.

New fused ops on the same path live in the same namespace
(``qkv_norm_rope_pack``, ``gated_residual``, ``gated_residual_norm_scale_shift``,
``gelu_tanh``, ``silu_mul``, ``timestep_embedding``, ``timestep_mlp``, ``rmsnorm_quant_fp8``,
``norm_scale_shift_quant_fp8``).
"""
import glob
import os
from typing import Optional

import torch

_here = os.path.dirname(__file__)
_so = glob.glob(os.path.join(_here, "_C*.so"))
if not _so:
    raise ImportError(f"joyomni_ops C extension not found in {_here}; build it first (python build.py)")
torch.ops.load_library(_so[0])

__all__ = [
    "fused_qk_norm_rope_3d_paired",
    "fused_joint_qkv_pack",
    "fused_cached_kv_pack",
    "fused_norm_scale_shift",
    "rmsnorm",
    "sgl_per_token_quant_fp8",
    "fp8_scaled_mm",
    "has_quant",
    "has_fp8",
    # new fused ops
    "qkv_norm_rope_pack",
    "gated_residual",
    "gated_residual_norm_scale_shift",
    "gelu_tanh",
    "silu_mul",
    "timestep_embedding",
    "timestep_mlp",
    "timestep_mlp_modulate",
    "fp8_scaled_mm_gated_residual",
    "fp8_scaled_mm_gelu_quant",
    "rmsnorm_quant_fp8",
    "norm_scale_shift_quant_fp8",
    "qkv_norm_rope_pack_into",
    "qkv_norm_rope_pack_host",
    "cached_k_rotate_into",
    "gelu_quant_fp8",
    "attn_merge",
    "gated_residual_norm_scale_shift_quant_fp8",
    "library_path",
]

_ops = torch.ops.joyomni_ops


def library_path() -> str:
    """Path of the C-ABI library (libjoyomni_b200.so) these ops call."""
    return os.path.join(_here, "libjoyomni_b200.so")


# ---------------------------------------------------------------- fake kernels
# As in the reference (joyomni_ops/__init__.py:36-101): FakeTensor kernels keep
# the native ops opaque inside one torch.compile graph.
@torch.library.register_fake("joyomni_ops::fused_qk_norm_rope_3d_paired")
def _fake_fused_qk_norm_rope_3d_paired(q, k, seq_len, num_heads, eps, q_weight, k_weight, cos, sin,
                                       k_pre_rope=None):
    return None


@torch.library.register_fake("joyomni_ops::fused_joint_qkv_pack")
def _fake_fused_joint_qkv_pack(img_q, img_k, img_v, txt_q, txt_k, txt_v, cached_k, cached_v,
                               txt_q_weight, txt_k_weight, eps):
    batch, img_len, heads, head_dim = img_q.shape
    txt_len = txt_q.shape[1]
    cache_len = cached_k.shape[1] if cached_k is not None else 0
    out_q = img_q.new_empty((batch, img_len + txt_len, heads, head_dim))
    out_k = img_q.new_empty((batch, cache_len + img_len + txt_len, heads, head_dim))
    return out_q, out_k, torch.empty_like(out_k)


@torch.library.register_fake("joyomni_ops::fused_cached_kv_pack")
def _fake_fused_cached_kv_pack(key0, value0, key1, value1, cos, sin):
    batch, len0, heads, head_dim = key0.shape
    len1 = key1.shape[1] if key1 is not None else 0
    out_key = key0.new_empty((batch, len0 + len1, heads, head_dim))
    return out_key, torch.empty_like(out_key)


@torch.library.register_fake("joyomni_ops::fused_norm_scale_shift")
def _fake_fused_norm_scale_shift(x, gamma, beta, scale, shift, norm_type, eps):
    return x.new_empty(x.shape)


@torch.library.register_fake("joyomni_ops::rmsnorm")
def _fake_rmsnorm(x, weight, eps):
    return x.new_empty(x.shape)


@torch.library.register_fake("joyomni_ops::sgl_per_token_quant_fp8")
def _fake_sgl_per_token_quant_fp8(input, output_q, output_s):
    return None


@torch.library.register_fake("joyomni_ops::fp8_scaled_mm")
def _fake_fp8_scaled_mm(mat_a, mat_b, scales_a, scales_b, out_dtype, bias=None):
    return mat_a.new_empty((mat_a.shape[0], mat_b.shape[1]), dtype=out_dtype)


@torch.library.register_fake("joyomni_ops::qkv_norm_rope_pack")
def _fake_qkv_norm_rope_pack(qkv, num_heads, q_weight, k_weight, cos, sin, eps, head_major, k_pre_rope=None):
    L = qkv.shape[0]
    D = qkv.shape[1] // (3 * num_heads)
    shape = (num_heads, L, D) if head_major else (L, num_heads, D)
    return qkv.new_empty(shape), qkv.new_empty(shape), qkv.new_empty(shape)


@torch.library.register_fake("joyomni_ops::qkv_norm_rope_pack_into")
def _fake_qkv_norm_rope_pack_into(qkv, num_heads, q_weight, k_weight, cos, sin, eps, q_out, k_out, v_out,
                                  k_pre_out=None):
    return None


@torch.library.register_fake("joyomni_ops::cached_k_rotate_into")
def _fake_cached_k_rotate_into(key, cos, sin, out_key):
    return None


@torch.library.register_fake("joyomni_ops::qkv_norm_rope_pack_host")
def _fake_qkv_norm_rope_pack_host(qkv_host, num_heads, q_weight, k_weight, cos, sin, eps, head_major, q_host, k_host,
                                  v_host, chunk_tokens):
    return None


@torch.library.register_fake("joyomni_ops::attn_merge")
def _fake_attn_merge(o_a, lse_a, o_b, lse_b):
    _, h, s, d = o_a.shape
    return o_a.new_empty((s, h, d))


@torch.library.register_fake("joyomni_ops::gelu_quant_fp8")
def _fake_gelu_quant_fp8(x):
    return (x.new_empty(x.shape, dtype=torch.float8_e4m3fn),
            x.new_empty((x.shape[0], 1), dtype=torch.float32))


@torch.library.register_fake("joyomni_ops::gated_residual_norm_scale_shift_quant_fp8")
def _fake_gated_residual_norm_scale_shift_quant_fp8(residual, x, gate, gamma, beta, scale, shift, norm_type, eps):
    n = residual.shape[-1]
    m = residual.numel() // n
    return (residual.new_empty(residual.shape), residual.new_empty((m, n), dtype=torch.float8_e4m3fn),
            residual.new_empty((m, 1), dtype=torch.float32))


@torch.library.register_fake("joyomni_ops::gated_residual")
def _fake_gated_residual(residual, x, gate):
    return residual.new_empty(residual.shape)


@torch.library.register_fake("joyomni_ops::gated_residual_norm_scale_shift")
def _fake_gated_residual_norm_scale_shift(residual, x, gate, gamma, beta, scale, shift, norm_type, eps):
    return residual.new_empty(residual.shape), residual.new_empty(residual.shape)


@torch.library.register_fake("joyomni_ops::gelu_tanh")
def _fake_gelu_tanh(x):
    return x.new_empty(x.shape)


@torch.library.register_fake("joyomni_ops::silu_mul")
def _fake_silu_mul(a, b):
    return a.new_empty(a.shape)


@torch.library.register_fake("joyomni_ops::timestep_embedding")
def _fake_timestep_embedding(t, dim, flip_sin_to_cos, downscale_freq_shift, scale, max_period):
    return t.new_empty((t.shape[0], dim), dtype=torch.float32)


@torch.library.register_fake("joyomni_ops::fp8_scaled_mm_gated_residual")
def _fake_fp8_scaled_mm_gated_residual(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, residual, gate):
    return mat_a.new_empty((mat_a.shape[0], mat_b.shape[1]), dtype=out_dtype)


@torch.library.register_fake("joyomni_ops::fp8_scaled_mm_gelu_quant")
def _fake_fp8_scaled_mm_gelu_quant(mat_a, mat_b, scales_a, scales_b, out_dtype, bias=None):
    m, n = mat_a.shape[0], mat_b.shape[1]
    return mat_a.new_empty((m, n), dtype=torch.float8_e4m3fn), mat_a.new_empty((m, 1), dtype=torch.float32)


@torch.library.register_fake("joyomni_ops::timestep_mlp")
def _fake_timestep_mlp(t, w1, b1, w2, b2, w3, b3, max_period):
    return (w1.new_empty((t.shape[0], w3.shape[0])), w1.new_empty((t.shape[0], w1.shape[0])))


@torch.library.register_fake("joyomni_ops::timestep_mlp_modulate")
def _fake_timestep_mlp_modulate(t, w1, b1, w2, b2, w3, b3, tables, max_period):
    proj = w3.shape[0]
    n_tables = tables.numel() // proj
    return w1.new_empty((t.shape[0], proj)), w1.new_empty((n_tables, t.shape[0], proj))


@torch.library.register_fake("joyomni_ops::rmsnorm_quant_fp8")
def _fake_rmsnorm_quant_fp8(x, weight, eps):
    return (x.new_empty(x.shape, dtype=torch.float8_e4m3fn),
            x.new_empty((x.shape[0], 1), dtype=torch.float32))


@torch.library.register_fake("joyomni_ops::norm_scale_shift_quant_fp8")
def _fake_norm_scale_shift_quant_fp8(x, gamma, beta, scale, shift, norm_type, eps):
    return (x.new_empty(x.shape, dtype=torch.float8_e4m3fn),
            x.new_empty((x.shape[0], 1), dtype=torch.float32))


# ---------------------------------------------------------------- wrappers (reference signatures)
def fused_qk_norm_rope_3d_paired(q, k, seq_len, num_heads, eps, q_weight, k_weight, cos, sin, k_pre_rope=None):
    """In-place fused RMSNorm(q,k) + 3D RoPE. q/k: [B, seq_len*num_heads, head_dim] bf16."""
    _ops.fused_qk_norm_rope_3d_paired(q, k, seq_len, num_heads, eps, q_weight, k_weight, cos, sin, k_pre_rope)


def fused_joint_qkv_pack(img_q, img_k, img_v, txt_q, txt_k, txt_v, cached_k, cached_v, txt_q_weight,
                         txt_k_weight, eps=1e-6):
    """Pack joint-attention Q/K/V and fuse text Q/K RMSNorm (bf16, B=1, D=128)."""
    return _ops.fused_joint_qkv_pack(img_q, img_k, img_v, txt_q, txt_k, txt_v, cached_k, cached_v,
                                     txt_q_weight, txt_k_weight, eps)


def fused_cached_kv_pack(key0, value0, key1, value1, cos, sin):
    """Rotate and pack one or two pre-RoPE cache segments (bf16, B=1, D=128)."""
    return _ops.fused_cached_kv_pack(key0, value0, key1, value1, cos, sin)


def _norm_code(norm_type: str) -> int:
    # joyomni_ops/__init__.py:129-132: unknown strings become -1, which the op rejects.
    return 0 if norm_type == "layer" else 1 if norm_type == "rms" else -1


def fused_norm_scale_shift(x, gamma, beta, scale, shift, norm_type, eps=1e-5):
    """Norm(x; gamma, beta) * (1 + scale) + shift. norm_type: 'layer' or 'rms'."""
    return _ops.fused_norm_scale_shift(x, gamma, beta, scale, shift, _norm_code(norm_type), eps)


def rmsnorm(x, weight, eps=1e-6):
    """(x / RMS(x)) * weight. x: [M, N], weight: [N]."""
    return _ops.rmsnorm(x, weight, eps)


def has_fp8() -> bool:
    return hasattr(_ops, "fp8_scaled_mm")


def has_quant() -> bool:
    return hasattr(_ops, "sgl_per_token_quant_fp8")


def sgl_per_token_quant_fp8(input, output_q, output_s):
    _ops.sgl_per_token_quant_fp8(input, output_q, output_s)


def fp8_scaled_mm(mat_a, mat_b, scales_a, scales_b, out_dtype, bias: Optional[torch.Tensor] = None):
    return _ops.fp8_scaled_mm(mat_a, mat_b, scales_a, scales_b, out_dtype, bias)


# ---------------------------------------------------------------- new fused ops
def qkv_norm_rope_pack(qkv, num_heads, q_weight, k_weight, cos, sin, eps=1e-6, head_major=True,
                       k_pre_rope: Optional[torch.Tensor] = None):
    """qkv [L, 3*H*D] (K H D order) -> q, k, v with per-head RMSNorm + RoPE on q/k.

    Outputs are [H, L, D] (head_major=True) or [L, H, D].  cos/sin: bf16 [L, D/2],
    or both None for text rows (no rotation; the model RMSNorm's double rounding).
    k_pre_rope, if given, receives the normalised k before rotation (same layout).
    """
    return _ops.qkv_norm_rope_pack(qkv, num_heads, q_weight, k_weight, cos, sin, eps, head_major, k_pre_rope)


def qkv_norm_rope_pack_into(qkv, num_heads, q_weight, k_weight, cos, sin, q_out, k_out, v_out, eps=1e-6,
                            k_pre_out=None):
    """qkv_norm_rope_pack writing into [L, H, D] views (e.g. slices of persistent Q / KV buffers);
    k_pre_out (same strides), if given, receives the normalised k before rotation."""
    _ops.qkv_norm_rope_pack_into(qkv, num_heads, q_weight, k_weight, cos, sin, eps, q_out, k_out, v_out, k_pre_out)


def cached_k_rotate_into(key, cos, sin, out_key):
    """RoPE of pre-RoPE cached keys [L, H, 128] into out_key [L, H, 128] (contiguous) with fp32
    full-width cos/sin [L, 128]: the keys of fused_cached_kv_pack, without the value copy."""
    _ops.cached_k_rotate_into(key, cos, sin, out_key)


def qkv_norm_rope_pack_host(qkv_host, num_heads, q_weight, k_weight, cos, sin, q_host, k_host, v_host, eps=1e-6,
                            head_major=True, chunk_tokens=675):
    """qkv_norm_rope_pack from a pinned host qkv [L, 3*H*D] into pinned host q/k/v
    ([H, L, D] head-major, else [L, H, D]); weights and cos/sin on the GPU.  Uploads,
    packs and downloads overlap chunk by chunk (chunk_tokens tokens each)."""
    _ops.qkv_norm_rope_pack_host(qkv_host, num_heads, q_weight, k_weight, cos, sin, eps, head_major, q_host, k_host,
                                 v_host, chunk_tokens)


def attn_merge(o_a, lse_a, o_b, lse_b):
    """Attention over the union of two disjoint key sets from the two partial results:
    o_a / o_b [1, H, S, D] with their log-sum-exps lse_a / lse_b fp32 [1, H, S] -> [S, H, D]."""
    return _ops.attn_merge(o_a, lse_a, o_b, lse_b)


def gelu_quant_fp8(x):
    """(q e4m3 [M, N], scale fp32 [M, 1]) of bf16(gelu_tanh(x))."""
    return _ops.gelu_quant_fp8(x)


def gated_residual_norm_scale_shift_quant_fp8(residual, x, gate, scale, shift, norm_type="layer", eps=1e-6,
                                              gamma=None, beta=None):
    """(h, q, s): h = residual + x*gate; (q, s) = FP8 quant of Norm(h)*(1+scale)+shift."""
    return _ops.gated_residual_norm_scale_shift_quant_fp8(residual, x, gate, gamma, beta, scale, shift,
                                                          _norm_code(norm_type), eps)


def gated_residual(residual, x, gate):
    """residual + x * gate (torch.addcmul(residual, x, gate)), gate broadcast over rows."""
    return _ops.gated_residual(residual, x, gate)


def gated_residual_norm_scale_shift(residual, x, gate, scale, shift, norm_type="layer", eps=1e-6,
                                    gamma=None, beta=None):
    """(h, Norm(h)*(1+scale)+shift) with h = residual + x*gate, in one pass."""
    return _ops.gated_residual_norm_scale_shift(residual, x, gate, gamma, beta, scale, shift,
                                                _norm_code(norm_type), eps)


def gelu_tanh(x):
    """F.gelu(x, approximate='tanh')."""
    return _ops.gelu_tanh(x)


def silu_mul(a, b):
    """silu(a) * b."""
    return _ops.silu_mul(a, b)


def timestep_embedding(t, dim=256, flip_sin_to_cos=True, downscale_freq_shift=0.0, scale=1.0,
                       max_period=10000.0):
    """Sinusoidal timestep projection (diffusers Timesteps), fp32 [B, dim]."""
    return _ops.timestep_embedding(t, dim, flip_sin_to_cos, downscale_freq_shift, scale, max_period)


def fp8_scaled_mm_gated_residual(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, residual, gate):
    """residual + gate * fp8_scaled_mm(...) with the residual in the GEMM epilogue
    (dit.py:536-538: the down-projection and ``fused_add_gate`` in one pass)."""
    return _ops.fp8_scaled_mm_gated_residual(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, residual, gate)


def fp8_scaled_mm_gelu_quant(mat_a, mat_b, scales_a, scales_b, out_dtype, bias: Optional[torch.Tensor] = None):
    """The MLP's fc1 -> GELU-tanh -> per-token FP8 (dit.py:508-513): (q [M, N] e4m3, s [M, 1] fp32),
    equal to gelu_quant_fp8(fp8_scaled_mm(...)) bit for bit; GELU and the row amax run in the
    GEMM epilogue, one more kernel quantises."""
    return _ops.fp8_scaled_mm_gelu_quant(mat_a, mat_b, scales_a, scales_b, out_dtype, bias)


def timestep_mlp(t, w1, b1, w2, b2, w3, b3, max_period=10000.0):
    """WanTimeTextImageEmbedding timestep branch (dit.py:574-579, 605-620):
    sinusoid(t) -> linear_1 -> SiLU -> linear_2 -> SiLU -> time_proj.
    Returns (vec bf16 [B, proj_dim], silu(temb) bf16 [B, dim])."""
    return _ops.timestep_mlp(t, w1, b1, w2, b2, w3, b3, max_period)


def timestep_mlp_modulate(t, w1, b1, w2, b2, w3, b3, tables, max_period=10000.0):
    """timestep_mlp plus every block's ModulateWan add (dit.py:103-116) in time_proj's epilogue.
    tables: bf16 [T, proj_dim] (each block's and stream's modulate_table, [6, D] flattened).
    Returns (vec bf16 [B, proj_dim], mods bf16 [T, B, proj_dim] = bf16(tables[t] + vec))."""
    return _ops.timestep_mlp_modulate(t, w1, b1, w2, b2, w3, b3, tables.reshape(-1, w3.shape[0]), max_period)


def rmsnorm_quant_fp8(x, weight, eps=1e-6):
    """(q e4m3 [M, N], scale fp32 [M, 1]) of bf16(rmsnorm(x) * weight)."""
    return _ops.rmsnorm_quant_fp8(x, weight, eps)


def norm_scale_shift_quant_fp8(x, gamma, beta, scale, shift, norm_type="layer", eps=1e-6):
    """(q e4m3 [M, N], scale fp32 [M, 1]) of bf16(Norm(x)*(1+scale)+shift)."""
    return _ops.norm_scale_shift_quant_fp8(x, gamma, beta, scale, shift, _norm_code(norm_type), eps)
