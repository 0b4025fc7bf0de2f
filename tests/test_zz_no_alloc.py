"""fh3cuda_matmul_noalloc_dev: the matmul for callers that cannot let a library allocate
device memory while they run (a host that budgets device memory up front, a process whose
memory belongs to another allocator, a loop that cannot afford cudaMalloc's device
synchronisation).  Its activation scratch is a fixed static device array instead.

Called through the C ABI and compared with the allocating entry point
(fh3cuda_matmul_dev) on calls in a row, so that each call runs over the previous
call's leftovers in the shared array, at row counts where the allocating entry point
takes its two-pass path; the library's allocation counters must not move across a
no-alloc call.  This file is collected last on purpose."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu


def _call(L, name, w, x, bias, n_out):
    import torch
    from fasth3inc_b200 import _lib
    y = torch.full((x.shape[0], n_out), float("nan"), dtype=torch.float32, device="cuda")
    d = _lib.Fh3CudaW(12, w.in_, w.out, w.data.data_ptr())
    rc = getattr(L, name)(ctypes.byref(d), x.data_ptr(), y.data_ptr(), x.shape[0],
                          None if bias is None else bias.data_ptr(),
                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _no_alloc_call(L, w, x, b, n_out):
    """The no-alloc entry point, checking the library's own allocation counters around it."""
    from fasth3inc_b200 import _lib
    before = _lib.alloc_stats()
    got = _call(L, "fh3cuda_matmul_noalloc_dev", w, x, b, n_out)
    assert _lib.alloc_stats() == before, "the no-alloc entry point allocated device memory"
    return got


def test_no_alloc_matches_allocating_entry_point(fh3):
    import torch
    from fasth3inc_b200 import _lib
    L = _lib.load()
    K, N = 1024, 300
    w = fh3.make_weights(N, K, seed=21, stream_id=5)
    g = torch.Generator(device="cuda").manual_seed(21)
    bias = torch.randn(N, device="cuda", generator=g)
    # two calls in a row: the larger first, so the second reads over stale rows;
    # 4096 rows is where the allocating entry point takes the two-pass path
    for M, b in ((4096, bias), (300, bias), (150, None), (4, bias)):
        x = torch.randn((M, K), device="cuda", generator=g)
        ref = _call(L, "fh3cuda_matmul_dev", w, x, b, N)
        got = _no_alloc_call(L, w, x, b, N)
        tol = 1e-5 if M <= 16 else 5e-3
        assert not np.isnan(got).any()
        assert rel_fro(got, ref) <= tol, M
    assert L.fh3cuda_device_status(None) == 0


def test_no_alloc_ignores_the_two_pass_switch(fh3, monkeypatch):
    """FH3CUDA_GEMM_KERNEL=two-pass sends the allocating entry point's GEMMs through a
    bf16 weight copy in scratch from 129 rows on; the no-alloc entry point keeps to the
    fused kernels and allocates nothing."""
    import torch
    from fasth3inc_b200 import _lib
    L = _lib.load()
    K, N = 512, 264
    w = fh3.make_weights(N, K, seed=22, stream_id=6)
    g = torch.Generator(device="cuda").manual_seed(22)
    monkeypatch.setenv("FH3CUDA_GEMM_KERNEL", "two-pass")
    for M in (2500, 700):
        x = torch.randn((M, K), device="cuda", generator=g)
        ref = _call(L, "fh3cuda_matmul_dev", w, x, None, N)
        got = _no_alloc_call(L, w, x, None, N)
        assert rel_fro(got, ref) <= 5e-3, M
    assert L.fh3cuda_device_status(None) == 0


def test_no_alloc_rejects_sizes_beyond_its_scratch(fh3):
    import torch
    from fasth3inc_b200 import _lib
    L = _lib.load()
    K = 5120
    w = fh3.make_weights(8, K, seed=1, stream_id=1)
    x = torch.zeros((1000, K), device="cuda")   # 5.1 M elements > 4 Mi
    y = torch.zeros((1000, 8), device="cuda")
    d = _lib.Fh3CudaW(12, K, 8, w.data.data_ptr())
    rc = L.fh3cuda_matmul_noalloc_dev(ctypes.byref(d), x.data_ptr(), y.data_ptr(), 1000, None, None)
    assert rc == -8
    assert b"exceeds the fixed scratch" in L.fh3cuda_last_error()
