"""The C ABI boundary, checked without a GPU: the library builds for sm_100a,
loads, exports every entry point include/fh3cuda.h declares, and reports
errors (no device, bad arguments) the way the header documents."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from conftest import HAS_GPU, ROOT

HEADER = os.path.join(ROOT, "include", "fh3cuda.h")


def _declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:fh3cuda|__wrap_fh3)_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from fasth3inc_b200 import _lib, build
    build.build()
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    names = _declared_functions()
    assert "fh3cuda_matmul" in names and "__wrap_fh3_matmul" in names and len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    from fasth3inc_b200._lib import EXPORTED
    assert sorted(EXPORTED) == names


def test_library_is_built_for_sm100a():
    from fasth3inc_b200 import build
    path = build.build()
    assert os.path.getsize(path) > 100_000
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.NVCC_FLAGS)


def test_row_bytes_matches_reference_rule(lib, oracle):
    for n in (1, 255, 256, 257, 5120, 5376, 13824, 14336):
        assert lib.fh3cuda_row_bytes(12, n) == oracle.row_bytes(12, n) == ((n + 255) // 256) * 144
        assert lib.fh3cuda_row_bytes(0, n) == 4 * n
    assert lib.fh3cuda_row_bytes(12, 0) == 0
    for t in (1, 30, 8, 10, 11, 13, 14):      # every other format fh3_dequant expands
        for n in (32, 256, 1000, 5376):
            assert lib.fh3cuda_row_bytes(t, n) == oracle.row_bytes(t, n) > 0
    for t in (2, 3, 6, 7, 9, 15, 99):         # row sizes without an expander in fh3_dequant
        assert lib.fh3cuda_row_bytes(t, 256) == 0


def test_fh3w_layout_matches_reference_struct():
    from fasth3inc_b200._lib import Fh3CudaW
    # include/fh3/fh3.h:82-87: int type; int64_t in; int64_t out; const uint8_t *data;
    assert ctypes.sizeof(Fh3CudaW) == 32
    assert [getattr(Fh3CudaW, f).offset for f in ("type", "in_", "out", "data")] == [0, 8, 16, 24]


def test_status_codes_reuse_reference_values():
    text = open(HEADER).read()
    codes = dict(re.findall(r"#define (FH3_\w+)\s+\((-?\d+)\)", text))
    codes.update(dict(re.findall(r"#define (FH3_OK)\s+(\d+)", text)))
    # include/fh3/fh3.h:218-226
    assert codes["FH3_OK"] == "0" and codes["FH3_ERR"] == "-1"
    assert codes["FH3_E_NOMEM"] == "-7" and codes["FH3_E_INVALID"] == "-8"


@pytest.mark.skipif(HAS_GPU, reason="checks the no-device path")
def test_no_device_is_reported_not_hidden(lib):
    from fasth3inc_b200._lib import FH3CUDA_E_NODEV, Fh3CudaW
    assert lib.fh3cuda_init(0) == FH3CUDA_E_NODEV
    assert b"device" in lib.fh3cuda_last_error()
    # the void drop-in records the failure instead of computing anything on the CPU
    w = Fh3CudaW(12, 256, 1, None)
    x = (ctypes.c_float * 256)()
    y = (ctypes.c_float * 1)(123.0)
    lib.fh3cuda_matmul(ctypes.byref(w), x, y, 1, None)
    assert lib.fh3cuda_take_status() == FH3CUDA_E_NODEV
    assert lib.fh3cuda_take_status() == 0  # cleared
    assert y[0] == 123.0


@pytest.mark.skipif(HAS_GPU, reason="checks the no-device path")
def test_package_api_raises_without_gpu():
    import fasth3inc_b200 as f
    with pytest.raises(Exception):
        f.init(0)


def test_vsa_num_tiles_matches_oracle_geometry(oracle):
    """The host-side tile geometry of fh3cuda_vsa_num_tiles against the oracle's restatement of
    build_vsa_geometry (src/core/fh3_vsa.c:32-161), fallbacks included (no GPU needed)."""
    import fasth3inc_b200 as fh3
    rng = np.random.default_rng(3)
    for _ in range(300):
        T, A = (int(x) for x in rng.integers(0, 200, 2))
        gt, gh, gw = (int(x) for x in rng.integers(1, 13, 3))
        V = gt * gh * gw
        n = T + A + V + (int(rng.integers(0, 3)) if rng.random() < 0.1 else 0)   # sometimes a count mismatch
        if rng.random() < 0.1:
            gw += 1                                                               # sometimes a grid mismatch
        tile = int(rng.choice([16, 32, 64, 100]))
        seq = (n, T, A, V, gt, gh, gw)
        assert fh3.vsa_num_tiles(seq, tile) == oracle.vsa_tiles(seq, tile), (seq, tile)


def test_fh3cudaseq_matches_reference_fh3seq_prefix():
    from fasth3inc_b200._lib import Fh3CudaSeq
    # src/model/fh3_seq.h:31-38: seven leading ints of struct Fh3Seq
    assert ctypes.sizeof(Fh3CudaSeq) == 28
    assert [getattr(Fh3CudaSeq, f).offset for f in ("seq_len", "num_text", "num_audio", "num_video", "grid_t",
                                                     "grid_h", "grid_w")] == [0, 4, 8, 12, 16, 20, 24]
