"""The drop-in fh3_matmul replacement on HOST buffers (fh3cuda_matmul / __wrap_fh3_matmul).

Same checks as the reference's tests/unit/test_matmul.c on its own golden file,
through the C entry point a relinked fh3 binary would call.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import read_matmul_golden, rel_fro

pytestmark = pytest.mark.gpu
Q4K = 12


def test_golden_through_dropin(fh3):
    t, K, N, M, w, x, bias, y = read_matmul_golden()
    # M = 37 takes the tensor-core GEMM (tolerance 5e-3); the first 16 tokens the fp32 GEMV (1e-5)
    got = fh3.matmul_host(w, K, N, x, bias)
    assert rel_fro(got, y) <= 5e-3
    got16 = fh3.matmul_host(w, K, N, x[:16], bias)
    assert rel_fro(got16, y[:16]) <= 1e-5


def test_registered_weights_match_staged(fh3, oracle):
    from fasth3inc_b200 import _lib
    L = _lib.load()
    K, N, M = 1024, 300, 40
    w = oracle.make_weights(seed=3, stream=1, rows=N, n=K)
    x = oracle.rng_normal(3, 2, M * K).reshape(M, K)
    staged = fh3.matmul_host(w, K, N, x)
    dev = ctypes.c_void_p()
    assert L.fh3cuda_upload_weights(w.ctypes.data, w.nbytes, ctypes.byref(dev)) == 0
    try:
        resident = fh3.matmul_host(w, K, N, x)
    finally:
        assert L.fh3cuda_release_weights(w.ctypes.data) == 0
    assert np.array_equal(staged, resident)
    assert rel_fro(resident, oracle.matmul(Q4K, w, K, N, x)) <= 5e-3


def test_wrap_symbol_is_the_dropin(fh3, oracle):
    from fasth3inc_b200 import _lib
    L = _lib.load()
    K, N, M = 512, 33, 3
    w = oracle.make_weights(seed=4, stream=1, rows=N, n=K)
    x = oracle.rng_normal(4, 2, M * K).reshape(M, K)
    y = np.zeros((M, N), np.float32)
    d = _lib.Fh3CudaW(Q4K, K, N, w.ctypes.data)
    L.__wrap_fh3_matmul(ctypes.byref(d), x.ctypes.data, y.ctypes.data, M, None)
    assert L.fh3cuda_take_status() == 0
    assert rel_fro(y, oracle.matmul(Q4K, w, K, N, x)) <= 1e-5


def test_bad_arguments_are_recorded_not_silent(fh3):
    from fasth3inc_b200 import _lib
    L = _lib.load()
    y = np.full((1, 4), 5.0, np.float32)
    x = np.zeros((1, 256), np.float32)
    w = np.zeros(4 * 144, np.uint8)
    d = _lib.Fh3CudaW(Q4K, 256, 4, w.ctypes.data)
    L.fh3cuda_matmul(ctypes.byref(d), x.ctypes.data, y.ctypes.data, 0, None)  # n_tok = 0
    assert L.fh3cuda_take_status() == -8
    d2 = _lib.Fh3CudaW(2, 256, 4, w.ctypes.data)   # Q4_0: fh3_dequant has no expander for it
    L.fh3cuda_matmul(ctypes.byref(d2), x.ctypes.data, y.ctypes.data, 1, None)
    assert L.fh3cuda_take_status() == -8
    assert np.all(y == 5.0)
