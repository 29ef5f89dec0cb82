"""Build recipe for the sm_100a joyomni library (no torch JIT cache, all in-tree).

Produces, inside ``joyomni_ops/`` next to this file:

* ``libjoyomni_b200.so`` -- the C-ABI library (``include/joyomni_b200.h``): every
  CUDA kernel, compiled with ``nvcc -gencode arch=compute_100a,code=sm_100a``;
  no torch dependency, static cudart.
* ``_C.so`` -- the ``torch.ops.joyomni_ops`` registration shim
  (``csrc/torch_shim.cpp``), linked against ``libjoyomni_b200.so`` through an
  ``$ORIGIN`` rpath.

Run ``python build.py`` (or ``__graft_entry__.build()``).  Object files go to
``_build/``; a file is recompiled when it or any header is newer than its object.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
OUT = HERE / "joyomni_ops"
BUILD = HERE / "_build"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    f"-I{INCLUDE}", f"-I{CSRC}",
]
CU_SOURCES = ["common.cu", "rows.cu", "rows_bf16.cu", "rows_f16.cu", "rows_f32.cu", "qkv.cu", "elementwise.cu",
              "fp8_gemm.cu", "temb.cu", "host_io.cu", "attn.cu", "peer.cu"]
LIB = OUT / "libjoyomni_b200.so"
SHIM = OUT / "_C.so"


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")
    if r.stderr.strip() and os.environ.get("JO_BUILD_VERBOSE"):
        sys.stderr.write(r.stderr)


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def build_lib(jobs: int = 8) -> Path:
    BUILD.mkdir(exist_ok=True)
    OUT.mkdir(exist_ok=True)
    hdrs = _headers()
    objs = []
    todo = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if _stale(o, [s] + hdrs):
            todo.append([NVCC, *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(_run, todo))
    if todo or _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs),
              "-Xlinker", "--exclude-libs,ALL"])
    return LIB


def build_shim() -> Path:
    import torch
    from torch.utils import cpp_extension as ce

    src = CSRC / "torch_shim.cpp"
    if not _stale(SHIM, [src, LIB] + _headers()):
        return SHIM
    inc = [f"-I{p}" for p in ce.include_paths("cuda")] + [f"-I{INCLUDE}"]
    libdirs = [p for p in ce.library_paths("cuda")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-w", *inc, str(src), "-o", str(SHIM),
           *[f"-L{p}" for p in libdirs], f"-L{OUT}",
           "-ljoyomni_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-Wl,-rpath,$ORIGIN"]
    _run(cmd)
    return SHIM


def build(jobs: int = 8) -> None:
    build_lib(jobs)
    build_shim()


def clean() -> None:
    shutil.rmtree(BUILD, ignore_errors=True)
    for p in (LIB, SHIM):
        if p.exists():
            p.unlink()


if __name__ == "__main__":
    if "--clean" in sys.argv:
        clean()
    build()
    print(f"built {LIB.name} and {SHIM.name} in {OUT}")
