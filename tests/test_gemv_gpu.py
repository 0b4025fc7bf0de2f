"""The small-M GEMV kernels (1..16 tokens) against fh3_matmul.

Tolerance: relative Frobenius error <= 1e-5 for the fp32
GEMV path, checked against the reference's own outputs (tests/golden) and the
oracle (bitwise equal to fh3_matmul, tests/test_oracle.py) at the BASELINE shapes.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import read_matmul_golden, rel_fro

pytestmark = pytest.mark.gpu
Q4K = 12
TOL = 1e-5
_PATH = {"kernel": "fp32"}


@pytest.fixture(autouse=True, params=["matmul", "gemv"])
def gemv_path(request):
    """Every test runs through both entry points that reach the small-M kernel: the
    dispatcher (fh3cuda_matmul_dev, 1..16 tokens) and fh3cuda_gemv_q4k_dev."""
    _PATH["kernel"] = request.param
    return request.param


@pytest.fixture(autouse=True, params=["default", "tc", "mma-stream", "mma-cta", "mma-i8", "fp32"])
def gemv_kernel(request, monkeypatch):
    """...and on every GEMV kernel: the default choice (warp-level integer MMAs at 1-2 tokens
    and at 3-4 when out > in, tcgen05 otherwise), the tcgen05 kernel forced for every
    shape ("tc"), the warp-MMA kernels ("mma-stream": persistent stream-K for 1..2 tokens,
    CTA-per-tile otherwise; "mma-cta" forces CTA-per-tile; "mma-i8": the stream-K kernels on
    integer MMAs of the nibbles against activation digits, for 1..4 tokens) and the fp32
    CUDA-core kernel (FH3CUDA_GEMV_KERNEL=fp32)."""
    if request.param == "default":
        monkeypatch.delenv("FH3CUDA_GEMV_KERNEL", raising=False)
    else:
        monkeypatch.setenv("FH3CUDA_GEMV_KERNEL", request.param)
    return request.param


def _run(fh3, w_raw, K, N, x, bias=None):
    import torch
    w = fh3.Q4KWeight.from_bytes(w_raw, K, N)
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    bt = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias, dtype=np.float32)).cuda()
    y = fh3.matmul(w, xt, bt) if _PATH["kernel"] == "matmul" else fh3.gemv(w, xt, bt)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_reference_cases(fh3, golden_cases):
    seen = 0
    for name in sorted({k.split("/")[0] for k in golden_cases if k.startswith("k")}):
        K, N, M = (int(v) for v in golden_cases[f"{name}/dims"])
        if M > 16:
            continue
        y = _run(fh3, golden_cases[f"{name}/w"], K, N, golden_cases[f"{name}/x"],
                 golden_cases.get(f"{name}/bias"))
        assert rel_fro(y, golden_cases[f"{name}/y"]) <= TOL, name
        seen += 1
    assert seen >= 5


def test_reference_fp64_golden_first_16_tokens(fh3):
    t, K, N, M, w, x, bias, y = read_matmul_golden()
    got = _run(fh3, w, K, N, x[:16], bias)
    assert rel_fro(got, y[:16]) <= TOL


@pytest.mark.parametrize("K,N", [(5120, 5120), (5120, 13824), (13824, 5120)])
@pytest.mark.parametrize("M", [1, 2, 4, 16])
def test_baseline_shapes_vs_oracle(fh3, oracle, K, N, M):
    w = oracle.make_weights(seed=K + N, stream=1, rows=N, n=K)
    x = oracle.rng_normal(M, 2, M * K).reshape(M, K)
    ref = oracle.matmul(Q4K, w, K, N, x)
    got = _run(fh3, w, K, N, x)
    assert rel_fro(got, ref) <= TOL


@pytest.mark.parametrize("M", [3, 6, 16])
def test_large_super_block_against_zero_weights(fh3, oracle, M):
    """x of one super-block near 1e8 meets all-zero weights (d = dmin = 0 in every row's
    header), so y comes from the other super-blocks alone: their x must keep their own
    precision, i.e. x is scaled per super-block, not per token (integer planes up to 5
    tokens, f16 pieces from 6)."""
    K, N, b0 = 1280, 64, 2
    w = oracle.make_weights(seed=11, stream=1, rows=N, n=K).copy()
    nblk = K // 256
    rows = w.reshape(N, nblk, 144)
    rows[:, b0, 0:4] = 0  # fp16 d and dmin of super-block b0
    x = oracle.rng_normal(M, 12, M * K).reshape(M, K).astype(np.float32)
    x[:, b0 * 256:(b0 + 1) * 256] *= np.float32(1e8)
    ref = oracle.matmul(Q4K, w, K, N, x)
    got = _run(fh3, w, K, N, x)
    assert rel_fro(got, ref) <= TOL


def test_every_token_count_and_row_tail(fh3, oracle):
    K, N = 1280, 37  # N not a multiple of the rows-per-warp
    w = oracle.make_weights(seed=5, stream=1, rows=N, n=K)
    b = oracle.rng_normal(5, 9, N)
    for M in range(1, 17):
        x = oracle.rng_normal(5, 10 + M, M * K).reshape(M, K)
        for bias in (None, b):
            ref = oracle.matmul(Q4K, w, K, N, x, bias)
            got = _run(fh3, w, K, N, x, bias)
            assert rel_fro(got, ref) <= TOL, (M, bias is None)


@pytest.mark.parametrize("K,Ms", [(27136, (1,)), (27392, (1, 2)), (18432, (3, 4)), (18688, (3, 4))])
def test_shared_memory_bounds_of_the_integer_kernels(fh3, oracle, K, Ms):
    """K at and just past the sizes whose activation digits fit the integer kernels' shared
    memory (1 token: 106 super-blocks; 4 tokens: 72): past them the dispatch falls back to
    the next kernel with the same accuracy.  1-2 tokens take the integer kernels on every
    shape; 3-4 tokens do under the "mma-i8" parameter of the kernel fixture."""
    N = 72
    w = oracle.make_weights(seed=K, stream=1, rows=N, n=K)
    for M in Ms:
        x = oracle.rng_normal(K, M, M * K).reshape(M, K)
        assert rel_fro(_run(fh3, w, K, N, x), oracle.matmul(Q4K, w, K, N, x)) <= TOL, M


def test_single_row_single_block(fh3, oracle):
    w = oracle.make_weights(seed=6, stream=1, rows=1, n=256)
    x = oracle.rng_normal(6, 2, 256).reshape(1, 256)
    assert rel_fro(_run(fh3, w, 256, 1, x), oracle.matmul(Q4K, w, 256, 1, x)) <= TOL


def test_rejects_bad_arguments(fh3, oracle):
    import torch
    w = fh3.Q4KWeight.from_bytes(oracle.make_weights(1, 1, 4, 256), 256, 4)
    x = torch.zeros((17, 256), dtype=torch.float32, device="cuda")
    with pytest.raises(fh3.Fh3CudaError):
        fh3.gemv(w, x)  # more than 16 tokens is the GEMM's job
    bad = fh3.Q4KWeight(w.data, 300, 4)  # in not a multiple of 256
    with pytest.raises(fh3.Fh3CudaError):
        fh3.gemv(bad, x[:1, :256])


def test_activation_ranges_and_zero_groups(fh3, oracle):
    """Per-16-element scales of the integer path: huge, tiny, zero and mixed-magnitude rows."""
    K, N, M = 1024, 70, 4
    w = oracle.make_weights(seed=9, stream=1, rows=N, n=K)
    x = oracle.rng_normal(9, 2, M * K).reshape(M, K).astype(np.float32)
    x[0] *= 3.0e4          # large activations
    x[1] *= 1.0e-6         # tiny activations
    x[2, :512] = 0.0       # whole zero groups
    x[3, ::7] *= 1000.0    # mixed magnitudes inside groups
    ref = oracle.matmul(Q4K, w, K, N, x)
    got = _run(fh3, w, K, N, x)
    for t in range(M):
        assert rel_fro(got[t], ref[t]) <= TOL, t


def test_split_tiles_repeat_bitwise(fh3, oracle):
    """Tiles split between CTAs (stream-K) are summed in a fixed order: repeated calls
    give identical bits, and consecutive calls on other weights leave no state behind."""
    import torch
    K, N = 13824, 1000
    ws = [fh3.Q4KWeight.from_bytes(oracle.make_weights(seed=20 + i, stream=1, rows=N, n=K), K, N) for i in range(2)]
    for M in (1, 2, 3, 4, 5, 8, 16):
        x = torch.from_numpy(oracle.rng_normal(21, M, M * K).reshape(M, K).astype(np.float32)).cuda()
        runs = []
        for r in range(3):
            runs.append([fh3.gemv(w, x).cpu().numpy() for w in ws])
        for r in range(1, 3):
            for a, b in zip(runs[0], runs[r]):
                assert np.array_equal(a, b), (M, r)
        ref = oracle.matmul(Q4K, oracle.make_weights(seed=20, stream=1, rows=N, n=K), K, N, x.cpu().numpy())
        assert rel_fro(runs[0][0], ref) <= TOL, M


def test_fresh_weight_buffers_first_call(fh3, oracle):
    """The first call on a freshly uploaded weight buffer (its pages cold, its TMA loads
    unevenly timed) gives the same result as later calls: guards the stage hand-off of
    the tcgen05 kernel, whose generic-proxy reads of a stage precede its TMA refill."""
    import torch
    K, N = 13824, 5120
    w = oracle.make_weights(seed=K + N, stream=1, rows=N, n=K)
    for M in (3, 5, 9, 16):
        x = oracle.rng_normal(M + 7, 2, M * K).reshape(M, K).astype(np.float32)
        ref = oracle.matmul(Q4K, w, K, N, x)
        keep = []
        for trial in range(4):
            W = fh3.Q4KWeight.from_bytes(w, K, N)
            keep.append(W)
            got = fh3.gemv(W, torch.from_numpy(x).cuda()).cpu().numpy()
            assert rel_fro(got, ref) <= TOL, (M, trial)


def test_non_finite_activations(fh3, oracle):
    """An Inf or NaN activation makes every output of its token non-finite, as fh3_matmul's
    fp32 sums do (Inf times a weight, and 0 * Inf = NaN for a zero weight); the other
    tokens keep the usual accuracy."""
    K, N = 1280, 70
    w = oracle.make_weights(seed=13, stream=1, rows=N, n=K)
    for M in (1, 2, 3, 4, 5, 8, 16):
        x = oracle.rng_normal(13, M, M * K).reshape(M, K).astype(np.float32)
        x[0, 300] = np.inf
        bad = {0}
        if M > 2:
            x[2, 17] = np.nan
            bad.add(2)
        with np.errstate(invalid="ignore", over="ignore"):
            ref = oracle.matmul(Q4K, w, K, N, x)
        got = _run(fh3, w, K, N, x)
        for t in range(M):
            if t in bad:
                assert not np.isfinite(ref[t]).any(), (M, t)  # the reference's own behaviour
                assert not np.isfinite(got[t]).any(), (M, t)
            else:
                assert rel_fro(got[t], ref[t]) <= TOL, (M, t)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_dependent_chain_queued_equals_synchronised(fh3, oracle, M):
    """GEMVs whose x is the previous call's y, queued back to back (each launched as a
    programmatic dependent of the previous kernel, its weights requested before the wait),
    give the same bits as the same chain with a synchronisation after every call."""
    import torch
    dims = [1024, 2048, 1024, 1280, 1024]
    ws = [fh3.Q4KWeight.from_bytes(oracle.make_weights(seed=300 + i, stream=1, rows=dims[i + 1], n=dims[i]),
                                   dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    x0 = torch.from_numpy(oracle.rng_normal(301, M, M * dims[0]).reshape(M, dims[0]).astype(np.float32)).cuda()
    run = fh3.matmul if _PATH["kernel"] == "matmul" else fh3.gemv

    def chain(sync):
        outs, h = [], x0
        for w in ws:
            h = run(w, h)
            outs.append(h)
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return outs

    ref = chain(True)
    for _ in range(2):
        for a, b in zip(ref, chain(False)):
            assert torch.equal(a, b)
