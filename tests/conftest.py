"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import os
import struct
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs through libfh3cuda")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build
    build()
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference
    if not Reference.available():
        pytest.skip("reference objects (oracle/_ref) not built in this tree")
    return Reference()


@pytest.fixture(scope="session")
def golden_cases():
    return dict(np.load(os.path.join(GOLDEN, "ref_cases.npz")))


def read_q4k_golden():
    """tests/fixtures/quant/Q4_K.bin of the reference: <IIII> type, rows, cols, nbytes; raw; fp32."""
    with open(os.path.join(GOLDEN, "Q4_K.bin"), "rb") as f:
        b = f.read()
    t, rows, cols, nb = struct.unpack("<IIII", b[:16])
    raw = np.frombuffer(b[16:16 + nb], np.uint8).copy()
    ref = np.frombuffer(b[16 + nb:], np.float32).reshape(rows, cols).copy()
    return t, rows, cols, raw, ref


def read_matmul_golden():
    """tests/fixtures/quant/matmul_ref.bin: <IIIII> type, K, N, M, wbytes; W; x; bias; y (fp64 numpy)."""
    with open(os.path.join(GOLDEN, "matmul_ref.bin"), "rb") as f:
        b = f.read()
    t, K, N, M, wb = struct.unpack("<IIIII", b[:20])
    off = 20
    w = np.frombuffer(b[off:off + wb], np.uint8).copy(); off += wb
    x = np.frombuffer(b[off:off + 4 * M * K], np.float32).reshape(M, K).copy(); off += 4 * M * K
    bias = np.frombuffer(b[off:off + 4 * N], np.float32).copy(); off += 4 * N
    y = np.frombuffer(b[off:off + 4 * M * N], np.float32).reshape(M, N).copy()
    return t, K, N, M, w, x, bias, y


def read_rmsnorm_golden():
    """tests/fixtures/ops/rmsnorm.bin: <II f> n, dim, eps; x [n][dim]; w [dim]; ref [n][dim]."""
    with open(os.path.join(GOLDEN, "rmsnorm.bin"), "rb") as f:
        b = f.read()
    n, dim = struct.unpack("<II", b[:8])
    (eps,) = struct.unpack("<f", b[8:12])
    a = np.frombuffer(b[12:], np.float32)
    x = a[:n * dim].reshape(n, dim).copy()
    w = a[n * dim:n * dim + dim].copy()
    ref = a[n * dim + dim:n * dim + dim + n * dim].reshape(n, dim).copy()
    return n, dim, eps, x, w, ref


def read_rope3_golden():
    """tests/fixtures/ops/rope3.bin: <IIII> n, heads, head_dim, rot_dim; x; cos [n][rot]; sin; ref."""
    with open(os.path.join(GOLDEN, "rope3.bin"), "rb") as f:
        b = f.read()
    n, heads, hd, rot = struct.unpack("<IIII", b[:16])
    a = np.frombuffer(b[16:], np.float32)
    nx, nr = n * heads * hd, n * rot
    x = a[:nx].reshape(n, heads * hd).copy()
    c = a[nx:nx + nr].reshape(n, rot).copy()
    s = a[nx + nr:nx + 2 * nr].reshape(n, rot).copy()
    ref = a[nx + 2 * nr:nx + 2 * nr + nx].reshape(n, heads * hd).copy()
    return n, heads, hd, rot, x, c, s, ref


def close_like_reference(got, ref, tol=1e-5) -> bool:
    """check_close of the reference's tests/unit/test_ops.c:41-56: |a-r| / max(|r|, 1) <= tol."""
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    return bool(np.all(np.abs(got - ref) / np.maximum(np.abs(ref), 1.0) <= tol))


@pytest.fixture(scope="session")
def fh3():
    """The product package on cuda:0; the CUDA library must load (no fallback)."""
    if not HAS_GPU:
        pytest.skip("no CUDA device")
    import fasth3inc_b200 as f
    from fasth3inc_b200 import build
    build.build()
    f.init(0)
    return f


def rel_fro(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


VSA_FIXTURES = ("vsa_n784", "vsa_padded", "vsa_sparsity0")


def read_vsa_golden(name: str):
    """tests/fixtures/vsa/<name>.bin of the reference (tests/unit/test_vsa.c:56-133):
    <9I> n, T, A, V, grid_t, grid_h, grid_w, heads, head_dim; <f> sparsity; <I> has_gate;
    then q, k, v, [gate], ref, each [n][heads*head_dim] fp32.
    Returns (seq = (n, T, A, V, gt, gh, gw), heads, head_dim, sparsity, q, k, v, gate|None, ref)."""
    with open(os.path.join(GOLDEN, "vsa", name + ".bin"), "rb") as f:
        b = f.read()
    hdr = struct.unpack("<9I", b[:36])
    (sp,) = struct.unpack("<f", b[36:40])
    (has_gate,) = struct.unpack("<I", b[40:44])
    n, heads, hd = hdr[0], hdr[7], hdr[8]
    e = n * heads * hd
    arrs, off = [], 44
    for _ in range(5 if has_gate else 4):
        arrs.append(np.frombuffer(b, np.float32, e, off).reshape(n, heads * hd).copy())
        off += 4 * e
    assert off == len(b)
    q, k, v = arrs[:3]
    gate = arrs[3] if has_gate else None
    return tuple(hdr[:7]), heads, hd, sp, q, k, v, gate, arrs[-1]


def vsa_case(golden_cases, name: str):
    """A reference-computed fh3_vsa_attention case from ref_cases.npz (tests/golden/make_golden.py)."""
    p = f"vsa_{name}/"
    seq = tuple(int(x) for x in golden_cases[p + "seq"])
    heads, hd, tile = (int(x) for x in golden_cases[p + "cfg"])
    sp = float(golden_cases[p + "sparsity"][0])
    gate = golden_cases.get(p + "gate")
    return (seq, heads, hd, tile, sp, golden_cases[p + "q"], golden_cases[p + "k"], golden_cases[p + "v"], gate,
            golden_cases[p + "y"])


VSA_CASES = ("hd128_tied", "nogate_tile32", "tile100", "mismatch_allvideo", "badgrid")


def rel_l2(a, b) -> float:
    """Relative L2 (Frobenius) error as tests/unit/test_vsa.c:43-53 computes it (fp64 sums)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.sqrt(np.sum(b * b))
    num = np.sqrt(np.sum((a - b) ** 2))
    return float(num / den) if den > 0 else float(num)
