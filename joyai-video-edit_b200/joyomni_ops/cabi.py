"""ctypes binding of the C ABI in ``include/joyomni_b200.h``.

This is the binding a host without the torch shim uses (and what the parity
tests call directly): plain device pointers, sizes, element strides, dtype
codes and a ``cudaStream_t`` as an integer.  ``call(name, *args)`` raises
``RuntimeError`` with ``jo_last_error()`` on a non-zero status.
"""
from __future__ import annotations

import ctypes as C
import os

_LIB_PATH = os.path.join(os.path.dirname(__file__), "libjoyomni_b200.so")

JO_OK = 0
JO_ERR_INVALID = -1
JO_ERR_SHAPE = -2
JO_ERR_ALIGN = -3
JO_ERR_DTYPE = -4
JO_ERR_CUDA = -5
JO_ERR_UNSUPPORTED = -6

JO_F32, JO_F16, JO_BF16, JO_E4M3 = 0, 1, 2, 3
JO_NORM_LAYER, JO_NORM_RMS = 0, 1


class JoView4(C.Structure):
    """jo_view4: a [1, L, H, 128] bf16 view, element (l, h, d) at ptr[l*sl + h*sh + d]."""

    _fields_ = [("ptr", C.c_void_p), ("len", C.c_int64), ("stride_l", C.c_int64), ("stride_h", C.c_int64)]


P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int
U64 = C.c_uint64
F32 = C.c_float
PP = C.POINTER(C.c_void_p)
FP = C.POINTER(C.c_float)

# name -> argtypes (restype is int unless listed in _RESTYPES)
SIGNATURES = {
    "jo_abi_version": [],
    "jo_status_name": [I32],
    "jo_last_error": [],
    "jo_launch_count": [],
    "jo_device_fault_count": [C.POINTER(C.c_uint32)],
    "jo_rmsnorm": [P, I64, P, I64, P, I64, I64, I32, F32, P],
    "jo_norm_scale_shift": [P, I64, P, I64, P, P, P, P, I64, I64, I64, I64, I32, I32, F32, P],
    "jo_qk_norm_rope_3d_paired": [P, P, I64, I64, I64, I64, F32, P, P, P, P, P, P],
    "jo_joint_qkv_pack": [P, P, P] + [JoView4] * 8 + [P, P, I64, F32, P],
    "jo_cached_kv_pack": [P, P] + [JoView4] * 4 + [P, P, I64, P],
    "jo_per_token_quant_fp8": [P, I64, P, P, I64, I64, I64, I32, P],
    "jo_fp8_scaled_mm": [P, I64, P, I64, P, I64, P, P, P, I64, I64, I64, I32, P],
    "jo_fp8_scaled_mm_gated_residual": [P, I64, P, I64, P, I64, P, P, P, P, I64, P, I64, I64, I64, I32, P],
    "jo_fp8_scaled_mm_gelu_quant": [P, I64, P, P, I64, P, P, I64, P, I64, P, P, P, I64, I64, I64, I32, P],
    "jo_qkv_norm_rope_pack": [P, P, P, P, I64, I64, P, I64, I64, I64, I64, P, P, P, P, F32, P],
    "jo_gated_residual": [P, I64, P, I64, P, I64, P, I64, I64, I64, I64, I32, P],
    "jo_gated_residual_norm_scale_shift": [P, I64, P, I64, P, I64, P, I64, P, I64, I64, P, P, P, P, I64, I64,
                                           I64, I64, I32, I32, F32, P],
    "jo_gelu_tanh": [P, P, I64, I32, P],
    "jo_silu_mul": [P, I64, P, I64, P, I64, I64, I64, I32, P],
    "jo_timestep_embedding": [P, P, I64, I64, I32, F32, F32, F32, P],
    "jo_timestep_mlp": [P, P, I64, P, P, I64, I64, P, P, P, P, I64, P, I64, F32, P],
    "jo_timestep_mlp_noalloc": [P, P, I64, P, P, I64, I64, P, P, P, P, I64, F32, P],
    "jo_timestep_mlp_modulate": [P, P, P, I64, P, I64, P, P, I64, I64, P, P, P, P, I64, P, I64, F32, P],
    "jo_qkv_norm_rope_pack_host": [P, P, P, I64, I64, P, P, P, P, P, I64, I64, I64, P, P, P, P, F32, I64, P, P, P],
    "jo_attn_merge": [P, I64, I64, P, I64, I64, P, I64, I64, P, I64, I64, P, I64, I64, I64, I64, I64, I32, P],
    "jo_rmsnorm_quant_fp8": [P, I64, P, P, I64, P, I64, I64, I32, F32, P],
    "jo_norm_scale_shift_quant_fp8": [P, I64, P, P, I64, P, P, P, P, I64, I64, I64, I64, I32, I32, F32, P],
    "jo_gelu_quant_fp8": [P, I64, P, P, I64, I64, I64, I32, P],
    "jo_gated_residual_norm_scale_shift_quant_fp8": [P, I64, P, I64, P, P, I64, P, I64, P, I64, I64, P, P, P, P,
                                                     I64, I64, I64, I64, I32, I32, F32, P],
    "jo_ipc_alloc": [I64, PP],
    "jo_ipc_free": [P],
    "jo_ipc_handle": [P, P],
    "jo_ipc_open": [P, PP],
    "jo_ipc_close": [P],
    "jo_peer_signal": [P, I32, U64, P],
    "jo_peer_wait": [P, I32, I32, U64, P],
    "jo_peer_copy": [P, P, I64, P],
}
JO_IPC_HANDLE_BYTES = 64
_RESTYPES = {"jo_status_name": C.c_char_p, "jo_last_error": C.c_char_p, "jo_launch_count": C.c_uint64}

_lib = None


def lib() -> C.CDLL:
    """Load libjoyomni_b200.so once and declare every entry point."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise ImportError(f"{_LIB_PATH} not found; build it first (python build.py)")
        L = C.CDLL(_LIB_PATH)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, C.c_int)
        _lib = L
    return _lib


def last_error() -> str:
    return lib().jo_last_error().decode()


def call(name: str, *args) -> None:
    """Call entry point ``name``; raise RuntimeError on a non-zero status."""
    status = getattr(lib(), name)(*args)
    if status != JO_OK:
        raise RuntimeError(f"{name}: {lib().jo_status_name(status).decode()}: {last_error()}")


def status_of(name: str, *args) -> int:
    """Call entry point ``name`` and return its raw status (no raise)."""
    return getattr(lib(), name)(*args)


def launch_count() -> int:
    return int(lib().jo_launch_count())


def device_fault_count() -> int:
    """Bounded-wait expiries recorded on the current device since the last call."""
    n = C.c_uint32(0)
    call("jo_device_fault_count", C.byref(n))
    return int(n.value)


# ------------------------------------------------------------------ torch helpers
def ptr(t) -> int:
    return t.data_ptr() if t is not None else None


def fptr(t):
    return C.cast(C.c_void_p(t.data_ptr()), FP) if t is not None else None


def stream(device=None) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt) -> int:
    import torch

    return {torch.float32: JO_F32, torch.float16: JO_F16, torch.bfloat16: JO_BF16,
            torch.float8_e4m3fn: JO_E4M3}[dt]


def view4(t) -> JoView4:
    """jo_view4 of a [1, L, H, D] tensor (or an empty view for None)."""
    if t is None:
        return JoView4(None, 0, 0, 0)
    return JoView4(t.data_ptr(), t.shape[1], t.stride(1), t.stride(2))
