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

BUILD_DIR = os.path.join(PKG, "_build")   # one object per source (git- and gpurun-ignored)
COMPILE_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]
LINK_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static"]
NVCC_FLAGS = COMPILE_FLAGS + ["-shared", "-cudart", "static"]  # the one-command form, for reference


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


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None, jobs: int | None = None) -> str:
    """Compile every CUDA source into fasth3inc_b200/libfh3cuda.so: one object per source,
    compiled in parallel (only the sources, or all of them after a header or flag change,
    whose objects are out of date), then one link."""
    if not force and not _stale():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    os.makedirs(BUILD_DIR, exist_ok=True)
    flags = [*COMPILE_FLAGS, *(extra or []), "-I", os.path.join(ROOT, "include")]
    stamp = os.path.join(BUILD_DIR, "flags.txt")
    sig = " ".join(flags)
    same_flags = os.path.exists(stamp) and open(stamp).read() == sig
    hdr = max(os.path.getmtime(p) for p in [os.path.join(CSRC, h) for h in HEADERS] +
              [os.path.join(ROOT, "include", "fh3cuda.h")])
    objs = [os.path.join(BUILD_DIR, os.path.splitext(f)[0] + ".o") for f in SOURCES]

    def fresh(src, obj):
        return (not force and same_flags and os.path.exists(obj) and
                os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr))

    todo = [(os.path.join(CSRC, f), o) for f, o in zip(SOURCES, objs) if not fresh(os.path.join(CSRC, f), o)]

    def compile_one(item):
        src, obj = item
        cmd = [_nvcc(), *flags, "-c", "-o", obj + ".tmp", src]
        if verbose:
            print(" ".join(cmd))
        out = subprocess.run(cmd, capture_output=True, text=True)
        if out.returncode != 0:
            return src, out.stdout + out.stderr
        os.replace(obj + ".tmp", obj)
        return None, out.stdout + out.stderr

    with ThreadPoolExecutor(max_workers=jobs or max(1, min(len(todo), os.cpu_count() or 1))) as ex:
        results = list(ex.map(compile_one, todo))
    errors = [(src, log) for src, log in results if src is not None]
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(f"{src}:\n{log}" for src, log in errors))
    if verbose:
        for _, log in results:
            if log:
                print(log)
    with open(stamp, "w") as f:
        f.write(sig)
    cmd = [_nvcc(), *LINK_FLAGS, "-o", LIB + ".tmp", *objs]
    if verbose:
        print(" ".join(cmd))
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + out.stdout + out.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB)
