"""The drop-in proven from C99: fh3 callers linked with -Wl,--wrap=fh3_matmul against
libfh3cuda.so (the link recipe for the reference's static fh3_core archive,
CMakeLists.txt:33; include/fh3/fh3.h:107).

oracle/Makefile's `relink` target builds two such programs into oracle/_ref/ where the
reference tree exists: relink_check (this project's C harness, comparing each wrapped
fh3_matmul call with __real_fh3_matmul, the reference's CPU function in the same
program, and with the reference's golden file) and bench_matmul_gpu (the reference's own
benchmarks/bench_matmul.c, unmodified, whose fh3_matmul calls at :78 and :89 now run on
the GPU).  Neither program calls anything but fh3 functions: the drop-in sets its device
up on first use."""
from __future__ import annotations

import os
import re
import subprocess

import pytest

from conftest import GOLDEN, ROOT

pytestmark = pytest.mark.gpu
REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def _exe(name: str) -> str:
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built (make -C oracle REF=<reference tree> relink)")
    return path


def test_relinked_c_caller_matches_real_fh3_matmul(fh3):
    out = subprocess.run([_exe("relink_check"), os.path.join(GOLDEN, "matmul_ref.bin")], capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "relink ok" in out.stdout
    assert out.stdout.count(" ok") >= 10


def test_reference_benchmark_runs_on_the_gpu_through_the_wrap(fh3):
    out = subprocess.run([_exe("bench_matmul_gpu"), "256", "2"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "fh3cuda_matmul:" not in out.stderr          # the drop-in reported no failure
    m = re.search(r"Peak Speed:\s+([0-9.]+) GFLOP/s", out.stdout)
    assert m and float(m.group(1)) > 0.0, out.stdout
