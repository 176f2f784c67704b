"""Build recipe for the native pieces of b200_gemm_b200.

Compiles, in-tree, with nvcc for sm_100a only:
  b200_gemm_b200/lib/libb200gemm.so   the C-ABI library (include/b200gemm.h)
  b200_gemm_b200/lib/gemm_bench       a C++ driver with the reference bench's
                                      verify-then-time loop (matmul_b200.cu)
The library links the CUDA runtime statically and resolves driver entry
points at run time, so it loads on machines without a GPU driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libb200gemm.so"
BENCH_BIN = LIBDIR / "gemm_bench"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include")]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build b200_gemm_b200")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h*"))


def build_library(force: bool = False, verbose: bool = False) -> Path:
    LIBDIR.mkdir(parents=True, exist_ok=True)
    if force or _stale(LIB, _sources()):
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-shared", "-cudart", "static",
               "-o", str(LIB), str(CSRC / "b200gemm.cu")]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
    return LIB


def build_bench(force: bool = False) -> Path:
    lib = build_library(force=force)
    src = CSRC / "gemm_bench.cu"
    if src.exists() and (force or _stale(BENCH_BIN, [src, lib])):
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-o", str(BENCH_BIN), str(src),
               "-L", str(LIBDIR), "-lb200gemm", "-Xlinker", "-rpath,$ORIGIN", "-lcublasLt"]
        subprocess.run(cmd, check=True)
    return BENCH_BIN


def build_all(force: bool = False) -> None:
    build_library(force=force)
    build_bench(force=force)


if __name__ == "__main__":
    import sys

    build_all(force="--force" in sys.argv)
    print(LIB)
