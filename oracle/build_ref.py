"""Build recipe for oracle/_ref/libjoyomni_ref.so -- test infrastructure only.

Compiles the reference's own light CUDA kernels, unmodified and where they lie in
the reference checkout (joyomni_ops/csrc/{rmsnorm, fused_norm_scale_shift,
fused_qknorm_rope_3d_kernel, fused_joint_qkv_pack, per_token_quant_fp8}.cu), with
nvcc for sm_100a, plus oracle/ref_ops.cpp, which registers them as
torch.ops.joyomni_ref.* (a namespace of their own, so they load beside this
repository's torch.ops.joyomni_ops.*).  The reference's build system is not used;
its FP8 GEMM (fp8_gemm.cu) needs CUTLASS at a pinned tag that is not available
here and is not built.  Outputs go to oracle/_ref/ only.

    python oracle/build_ref.py [REFERENCE_ROOT]

REFERENCE_ROOT defaults to $JOYOMNI_REFERENCE, else a ``reference`` directory
beside the repository.  Without a reference checkout nothing is built (the GPU
box uses the library built here, which travels with the repository).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libjoyomni_ref.so"
KERNELS = ["rmsnorm", "fused_norm_scale_shift", "fused_qknorm_rope_3d_kernel", "fused_joint_qkv_pack",
           "per_token_quant_fp8"]
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def reference_root(arg: str | None = None) -> Path | None:
    for cand in (arg, os.environ.get("JOYOMNI_REFERENCE"), str(HERE.parent.parent / "reference")):
        if cand and (Path(cand) / "joyomni_ops" / "csrc" / "rmsnorm.cu").is_file():
            return Path(cand)
    return None


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(" ".join(cmd[:2]) + " ... failed:\n" + (r.stdout + r.stderr)[-4000:])


def _stale(target: Path, deps: list[Path]) -> bool:
    return not target.exists() or any(d.stat().st_mtime > target.stat().st_mtime for d in deps)


def build(ref: Path | None = None, jobs: int = 8) -> Path | None:
    """Compile the library if a reference checkout is present; returns its path, or None."""
    ref = reference_root(str(ref) if ref else None)
    if ref is None:
        return None
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce

    csrc, inc = ref / "joyomni_ops" / "csrc", ref / "joyomni_ops" / "include"
    objdir = OUT / "obj"
    objdir.mkdir(parents=True, exist_ok=True)
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"
    incs = [f"-I{p}" for p in ce.include_paths("cuda")] + [f"-I{sysconfig.get_paths()['include']}", f"-I{inc}"]
    nvcc = [os.path.join(CUDA_HOME, "bin", "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-O3",
            "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", abi, *incs]
    objs, todo = [], []
    for k in KERNELS:
        src, obj = csrc / f"{k}.cu", objdir / f"{k}.o"
        objs.append(obj)
        if _stale(obj, [src]):
            todo.append(nvcc + ["-c", str(src), "-o", str(obj)])
    reg_src, reg_obj = HERE / "ref_ops.cpp", objdir / "ref_ops.o"
    objs.append(reg_obj)
    if _stale(reg_obj, [reg_src]):
        todo.append(["g++", "-O2", "-std=c++17", "-fPIC", abi, "-w", *incs, "-c", str(reg_src), "-o", str(reg_obj)])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(_run, todo))
    if todo or _stale(LIB, objs):
        libdirs = [f"-L{p}" for p in ce.library_paths("cuda")]
        _run(["g++", "-shared", "-o", str(LIB), *map(str, objs), *libdirs,
              f"-L{os.path.join(CUDA_HOME, 'lib64')}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
              "-ltorch_cuda", "-lcudart"])
    return LIB


if __name__ == "__main__":
    path = build(Path(sys.argv[1]) if len(sys.argv) > 1 else None)
    print(f"built {path}" if path else "no reference checkout found: nothing built")
