"""Failure paths, made to happen without faulting the GPU.

* A bounded device-side wait that runs out: fh3cuda_wait_selftest_dev launches one
  thread that waits, through the same bounded mbarrier wait every kernel uses, on a
  barrier nobody arrives at.  The kernel must return, the status word must read
  FH3CUDA_E_TIMEOUT, and the context must stay usable.
* An allocation failure injected on the host: a scratch budget
  (fh3cuda_set_scratch_limit) smaller than a call needs.  The device-pointer entry
  point returns FH3_E_NOMEM and computes nothing; the void drop-in records it as its
  sticky status, where fh3_matmul would skip its tiles silently
  (src/core/fh3_ops.c:325-328).  Run in a fresh process so that no earlier test's
  scratch is already large enough.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, rel_fro

pytestmark = pytest.mark.gpu

FH3_E_NOMEM = -7
FH3CUDA_E_TIMEOUT = -21


def test_bounded_wait_gives_up_and_context_stays_usable(fh3, oracle):
    import torch
    from fasth3inc_b200 import _lib
    L = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    assert L.fh3cuda_device_status(s) == 0
    assert L.fh3cuda_wait_selftest_dev(50_000_000, s) == 0        # 50 ms limit
    assert L.fh3cuda_device_status(s) == FH3CUDA_E_TIMEOUT
    assert b"gave up" in L.fh3cuda_last_error()
    assert L.fh3cuda_device_status(s) == 0                         # read once, then cleared
    # the context still computes
    K, N, M = 512, 96, 40
    raw = oracle.make_weights(seed=7, stream=1, rows=N, n=K)
    w = fh3.Q4KWeight.from_bytes(raw, K, N, device="cuda:0")
    x = oracle.rng_normal(7, 2, M * K).reshape(M, K)
    y = fh3.matmul(w, torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_fro(y, oracle.matmul(12, raw, K, N, x)) <= 5e-3
    assert L.fh3cuda_device_status(s) == 0


def test_bad_wait_limits_are_rejected(fh3):
    from fasth3inc_b200 import _lib
    L = _lib.load()
    assert L.fh3cuda_wait_selftest_dev(0, None) == -8
    assert L.fh3cuda_wait_selftest_dev(5_000_000_000, None) == -8


_CHILD = r"""
import ctypes, json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import torch
import fasth3inc_b200 as fh3
from fasth3inc_b200 import _lib
from oracle.oracle import Oracle, rel_fro
fh3.init(0)
L = _lib.load()
o = Oracle()
K, N, M = 1024, 512, 2304          # 2304 rows: the two-pass GEMM and its bf16 weight copy
raw = o.make_weights(seed=8, stream=1, rows=N, n=K)
x = o.rng_normal(8, 2, M * K).reshape(M, K)
res = {}
calls0, held0 = _lib.alloc_stats()
_lib.set_scratch_limit(held0 + 4096)     # no room for any new scratch
w = fh3.Q4KWeight.from_bytes(raw, K, N, device="cuda:0")
xd = torch.from_numpy(x).cuda()
yd = torch.full((M, N), 7.0, device="cuda")
d = w.desc
res["dev_rc"] = L.fh3cuda_matmul_dev(ctypes.byref(d), xd.data_ptr(), yd.data_ptr(), M, None,
                                     torch.cuda.current_stream().cuda_stream)
res["dev_msg"] = L.fh3cuda_last_error().decode()
torch.cuda.synchronize()
res["y_untouched"] = bool(torch.all(yd == 7.0).item())
yh = np.full((M, N), 3.0, np.float32)
dh = _lib.Fh3CudaW(12, K, N, raw.ctypes.data)
L.fh3cuda_matmul(ctypes.byref(dh), x.ctypes.data, yh.ctypes.data, M, None)
res["sticky"] = L.fh3cuda_take_status()
res["sticky_after"] = L.fh3cuda_take_status()
res["host_y_untouched"] = bool(np.all(yh == 3.0))
res["held_within_limit"] = _lib.alloc_stats()[1] <= held0 + 4096
_lib.set_scratch_limit(0)
L.fh3cuda_matmul(ctypes.byref(dh), x.ctypes.data, yh.ctypes.data, M, None)
res["sticky_unlimited"] = L.fh3cuda_take_status()
res["err_unlimited"] = rel_fro(yh, o.matmul(12, raw, K, N, x))
print("RESULT " + json.dumps(res))
"""


def test_scratch_budget_gives_nomem_in_a_fresh_process(fh3):
    env = dict(os.environ)
    env.pop("FH3CUDA_GEMM_KERNEL", None)
    out = subprocess.run([sys.executable, "-c", _CHILD, ROOT], capture_output=True, text=True, timeout=600,
                         env=env)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-2000:]
    line = [ln for ln in out.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    r = json.loads(line[len("RESULT "):])
    assert r["dev_rc"] == FH3_E_NOMEM, r
    assert "exceed the limit" in r["dev_msg"], r
    assert r["y_untouched"], r
    assert r["sticky"] == FH3_E_NOMEM and r["sticky_after"] == 0, r
    assert r["host_y_untouched"], r
    assert r["held_within_limit"], r
    assert r["sticky_unlimited"] == 0, r
    assert r["err_unlimited"] <= 5e-3, r
