"""Build the native libraries of the MoE FFN grouped-GEMM path in-tree.

Outputs (git-ignored, shipped with the source tree):
  cutlass_op/bf16_grouped_mm/libmoe_gemm.so        C ABI (include/moe_gemm.h), sm_100a kernels
  cutlass_op/bf16_grouped_mm/_grouped_mm_ops.so    torch.library ops `grouped_mm::*` over that ABI

Only nvcc (for sm_100a) and g++ are used; no JIT cache outside the tree.  A target is rebuilt
when any of its sources or headers is newer than it.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
OUT_DIR = PKG_ROOT / "cutlass_op" / "bf16_grouped_mm"
LIB = OUT_DIR / "libmoe_gemm.so"
OPS = OUT_DIR / "_grouped_mm_ops.so"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = CUDA_HOME / "bin" / "nvcc"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_lib(verbose: bool = False, force: bool = False) -> Path:
    srcs = sorted(CSRC.glob("*.cu"))
    deps = srcs + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    if force or _newer(LIB, deps):
        cmd = [NVCC, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
               "-Xcompiler", "-fPIC", "-shared", f"-I{INCLUDE}", f"-I{CSRC}", "-o", LIB, *srcs]
        _run(cmd, verbose)
    return LIB


def build_ops(verbose: bool = False, force: bool = False) -> Path:
    import torch
    import torch.utils.cpp_extension as ext

    src = CSRC / "torch_ops.cpp"
    deps = [src, LIB, *sorted(INCLUDE.glob("*.h"))]
    if force or _newer(OPS, deps):
        incs = [f"-I{p}" for p in ext.include_paths(device_type="cuda")]
        libdirs = ext.library_paths(device_type="cuda")
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
               "-DTORCH_API_INCLUDE_EXTENSION_H", *incs, f"-I{INCLUDE}", src, "-o", OPS,
               *[f"-L{d}" for d in libdirs], f"-L{OUT_DIR}",
               "-lmoe_gemm", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lcudart",
               "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{d}" for d in libdirs]]
        _run(cmd, verbose)
    return OPS


def build(verbose: bool = False, force: bool = False) -> None:
    build_lib(verbose, force)
    build_ops(verbose, force)


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
