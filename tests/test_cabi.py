"""C-ABI library and torch-op boundary checks that need no GPU.

* libjoyomni_b200.so loads and exports every entry point include/*.h declares,
  and the ctypes binding declares each of them.
* _C.so registers the seven reference schemas verbatim
  (joyomni_ops/csrc/pybind.cpp:52-75) plus the new fused ops.
* The ops have no CPU implementation: CPU tensors raise instead of silently
  falling back, and the C ABI refuses to run without an sm_100 device.
* FakeTensor registrations produce the reference output shapes.
"""
import ctypes
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent

REFERENCE_SCHEMAS = {
    "fused_qk_norm_rope_3d_paired": "fused_qk_norm_rope_3d_paired(Tensor! q, Tensor! k, int seq_len, "
                                    "int num_heads, float eps, Tensor q_weight, Tensor k_weight, Tensor cos, "
                                    "Tensor sin, Tensor? k_pre_rope) -> ()",
    "fused_joint_qkv_pack": "fused_joint_qkv_pack(Tensor img_q, Tensor img_k, Tensor img_v, Tensor txt_q, "
                            "Tensor txt_k, Tensor txt_v, Tensor? cached_k, Tensor? cached_v, Tensor txt_q_weight, "
                            "Tensor txt_k_weight, float eps) -> (Tensor, Tensor, Tensor)",
    "fused_cached_kv_pack": "fused_cached_kv_pack(Tensor key0, Tensor value0, Tensor? key1, Tensor? value1, "
                            "Tensor cos, Tensor sin) -> (Tensor, Tensor)",
    "fused_norm_scale_shift": "fused_norm_scale_shift(Tensor x, Tensor? gamma_opt, Tensor? beta_opt, Tensor scale, "
                              "Tensor shift, int norm_type, float eps) -> Tensor",
    "rmsnorm": "rmsnorm(Tensor x, Tensor weight, float eps) -> Tensor",
    "sgl_per_token_quant_fp8": "sgl_per_token_quant_fp8(Tensor input, Tensor! output_q, "
                               "Tensor! output_s) -> ()",
    "fp8_scaled_mm": "fp8_scaled_mm(Tensor mat_a, Tensor mat_b, Tensor scales_a, Tensor scales_b, "
                     "ScalarType out_dtype, Tensor? bias) -> Tensor",
}


def header_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        names |= set(re.findall(r"^JO_API\s+[\w\s\*]+?\b(jo_\w+)\s*\(", h.read_text(), flags=re.M))
    return names


def test_header_parses():
    names = header_symbols()
    assert "jo_rmsnorm" in names and "jo_fp8_scaled_mm" in names and len(names) >= 19


def test_library_exports_every_declared_symbol(cabi):
    lib = ctypes.CDLL(cabi._LIB_PATH)
    missing = [n for n in header_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_ctypes_binding_covers_header(cabi):
    assert header_symbols() == set(cabi.SIGNATURES), "cabi.SIGNATURES out of sync with include/*.h"


def header_arity():
    """Parameter count of every entry point, read from the declarations in include/*.h."""
    arity = {}
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^JO_API\s+[\w\s\*]+?\b(jo_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.M | re.S):
            params = m.group(2).strip()
            arity[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return arity


def test_ctypes_binding_arity_matches_header(cabi):
    arity = header_arity()
    assert set(arity) == header_symbols()
    wrong = {n: (len(cabi.SIGNATURES[n]), a) for n, a in arity.items() if len(cabi.SIGNATURES[n]) != a}
    assert not wrong, f"ctypes argument count differs from the header (binding, header): {wrong}"


def test_abi_info(cabi):
    L = cabi.lib()
    assert L.jo_abi_version() == 1
    assert L.jo_status_name(0) == b"JO_OK"
    assert L.jo_status_name(-6) == b"JO_ERR_UNSUPPORTED"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU refusal")
def test_cabi_refuses_without_device(cabi):
    # No GPU here: the entry point must fail with a status, not run anything.
    st = cabi.status_of("jo_rmsnorm", None, 0, None, 0, None, 4, 8, cabi.JO_BF16, 1e-6, None)
    assert st in (cabi.JO_ERR_CUDA, cabi.JO_ERR_UNSUPPORTED)
    assert cabi.last_error()


def test_reference_schemas_verbatim(jo):
    for name, schema in REFERENCE_SCHEMAS.items():
        got = getattr(torch.ops.joyomni_ops, name).default._schema
        want = torch._C.parse_schema("joyomni_ops::" + schema)
        assert got == want, f"{name}: {got} != {want}"


def test_new_ops_registered(jo):
    for name in ("qkv_norm_rope_pack", "gated_residual", "gated_residual_norm_scale_shift", "gelu_tanh",
                 "silu_mul", "timestep_embedding", "rmsnorm_quant_fp8", "norm_scale_shift_quant_fp8"):
        assert hasattr(torch.ops.joyomni_ops, name)


def test_feature_probes(jo):
    assert jo.has_fp8() and jo.has_quant()


def test_no_cpu_fallback(jo):
    x = torch.randn(4, 64, dtype=torch.bfloat16)
    w = torch.ones(64, dtype=torch.bfloat16)
    with pytest.raises((NotImplementedError, RuntimeError)):
        jo.rmsnorm(x, w, 1e-6)
    with pytest.raises((NotImplementedError, RuntimeError)):
        jo.gelu_tanh(x)


def test_fake_shapes(jo):
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        qkv = torch.empty(100, 3 * 4 * 128, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(128, dtype=torch.bfloat16, device="cuda")
        cs = torch.empty(100, 64, dtype=torch.bfloat16, device="cuda")
        q, k, v = jo.qkv_norm_rope_pack(qkv, 4, w, w, cs, cs)
        assert q.shape == (4, 100, 128) and v.shape == (4, 100, 128)
        img = torch.empty(1, 17, 4, 128, dtype=torch.bfloat16, device="cuda")
        txt = torch.empty(1, 11, 4, 128, dtype=torch.bfloat16, device="cuda")
        cache = torch.empty(1, 9, 4, 128, dtype=torch.bfloat16, device="cuda")
        oq, ok, ov = jo.fused_joint_qkv_pack(img, img, img, txt, txt, txt, cache, cache, w, w)
        assert oq.shape == (1, 28, 4, 128) and ok.shape == (1, 37, 4, 128) and ov.shape == ok.shape
        a = torch.empty(64, 128, dtype=torch.float8_e4m3fn, device="cuda")
        b = torch.empty(256, 128, dtype=torch.float8_e4m3fn, device="cuda").t()
        d = jo.fp8_scaled_mm(a, b, torch.empty(64, 1, device="cuda"), torch.empty(1, 256, device="cuda"),
                             torch.bfloat16)
        assert d.shape == (64, 256) and d.dtype == torch.bfloat16
        x = torch.empty(32, 3072, dtype=torch.bfloat16, device="cuda")
        qq, ss = jo.rmsnorm_quant_fp8(x, torch.empty(3072, dtype=torch.bfloat16, device="cuda"))
        assert qq.dtype == torch.float8_e4m3fn and ss.shape == (32, 1)


def test_norm_type_mapping(jo):
    assert jo._norm_code("layer") == 0 and jo._norm_code("rms") == 1 and jo._norm_code("bogus") == -1


def header_params():
    """name -> list of C parameter types, from every JO_API declaration in include/*.h."""
    out = {}
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", " ", h.read_text(), flags=re.S)
        for m in re.finditer(r"JO_API\s+[\w\s\*]+?\b(jo_\w+)\s*\(([^)]*)\)\s*;", text):
            params = [p.strip() for p in m.group(2).split(",") if p.strip()]
            if params == ["void"]:
                params = []
            out[m.group(1)] = [re.sub(r"\s+\w+$", "", p).replace(" ", "") for p in params]
    return out


def ctype_kind(c_type):
    if c_type.endswith("*"):
        return "ptr"
    return {"int64_t": "i64", "int": "i32", "float": "f32", "jo_view4": "view4", "uint32_t": "u32",
            "uint64_t": "u64"}[c_type]


def test_ctypes_argument_kinds_match_header(cabi):
    """Every ctypes argtype list has the header's arity and kinds (catches ABI drift)."""
    import ctypes as C

    kind = {C.c_void_p: "ptr", C.c_int64: "i64", C.c_int32: "i32", C.c_int: "i32", C.c_float: "f32",
            C.c_uint64: "u64", cabi.JoView4: "view4"}
    decls = header_params()
    assert set(decls) == set(cabi.SIGNATURES)
    for name, c_params in decls.items():
        got = [kind.get(t, "ptr" if isinstance(t, type) and issubclass(t, C._Pointer) else repr(t))
               for t in cabi.SIGNATURES[name]]
        want = [ctype_kind(p) for p in c_params]
        assert got == want, f"{name}: ctypes {got} vs header {want}"
