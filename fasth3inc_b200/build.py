"""Build libfh3cuda.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m fasth3inc_b200.build          # or fasth3inc_b200.build.build()
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libfh3cuda.so")
SOURCES = ["api.cu", "dequant.cu", "gemv.cu", "gemv_mma.cu", "gemv_tc.cu", "gemm.cu", "ops.cu", "attention.cu", "attention_tc.cu", "attention_f32.cu",
           "vsa.cu", "vsa_tc.cu", "trunk_io.cu", "dit.cu", "gen.cu", "noalloc.cu", "formats.cu"]
HEADERS = ["common.cuh", "flash.cuh", "formats.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared", "-cudart", "static",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "fh3cuda.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compile every CUDA source into fasth3inc_b200/libfh3cuda.so."""
    if not force and not _stale():
        return LIB
    cmd = [_nvcc(), *NVCC_FLAGS, *(extra or []), "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp"]
    cmd += [os.path.join(CSRC, f) for f in SOURCES]
    if verbose:
        print(" ".join(cmd))
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + out.stdout + out.stderr)
    if verbose and (out.stdout or out.stderr):
        print(out.stdout + out.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB)
