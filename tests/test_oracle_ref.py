"""The reference's own light CUDA kernels, built from its sources into oracle/_ref/
(oracle/build_ref.py), load beside this repository's ops and expose the reference
schemas (joyomni_ops/csrc/pybind.cpp:52-69) under torch.ops.joyomni_ref.

CPU-only checks (no kernel runs): the library loads, every op is registered with
the same schema as the drop-in op of the same name, and CPU tensors raise.
Skipped where the library was not built (no reference checkout at build time).
"""
from pathlib import Path

import pytest
import torch

REF_LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libjoyomni_ref.so"
OPS = ["rmsnorm", "fused_norm_scale_shift", "fused_qk_norm_rope_3d_paired", "fused_joint_qkv_pack",
       "fused_cached_kv_pack", "sgl_per_token_quant_fp8"]

pytestmark = pytest.mark.skipif(not REF_LIB.exists(), reason="oracle/_ref not built (no reference checkout)")


@pytest.fixture(scope="module")
def ref(jo):
    torch.ops.load_library(str(REF_LIB))
    return torch.ops.joyomni_ref


def test_reference_kernels_register_the_drop_in_schemas(ref):
    for name in OPS:
        theirs = str(getattr(ref, name).default._schema).replace("joyomni_ref::", "")
        ours = str(getattr(torch.ops.joyomni_ops, name).default._schema).replace("joyomni_ops::", "")
        assert theirs == ours, name


def test_reference_kernels_have_no_cpu_path(ref):
    x = torch.zeros(2, 8, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        ref.rmsnorm(x, torch.ones(8, dtype=torch.bfloat16), 1e-6)
