"""The weight formats other than Q4_K (the text encoder's Q5_K / Q6_K, the F16 globals,
and every other format fh3_dequant expands) on the GPU.

Dequantisation is bit-exact with the reference (its gguf fixtures and the oracle, which is
bitwise equal to fh3_dequant; NaN payloads of random fp16 scales compared as NaN).  The
matmul forms fh3_dequant's fp32 weights and contracts them at fp32 accuracy: up to 16
tokens on the CUDA cores, above that on the tcgen05 tensor cores as four bf16 products of
split operands.  Relative Frobenius error <= 1e-5 against fh3_matmul (the oracle, and the
reference's own outputs in tests/golden)."""
from __future__ import annotations

import os
import struct

import numpy as np
import pytest

from conftest import GOLDEN, rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-5
FORMATS = {"F16": 1, "BF16": 30, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}
# byte offsets of the fp16 scale fields of one block, and the block's (bytes, weights)
SCALES = {8: ((0,), 34, 32), 10: ((80, 82), 84, 256), 11: ((108,), 110, 256), 12: ((0, 2), 144, 256),
          13: ((0, 2), 176, 256), 14: ((208,), 210, 256)}


def _fixture(name):
    with open(os.path.join(GOLDEN, f"{name}.bin"), "rb") as f:
        b = f.read()
    t, rows, cols, nb = struct.unpack("<IIII", b[:16])
    return t, rows, cols, np.frombuffer(b[16:16 + nb], np.uint8).copy(), \
        np.frombuffer(b[16 + nb:], np.float32).reshape(rows, cols).copy()


def _same(a, b):
    nan = np.isnan(a)
    return np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


def _weights(oracle, t, rows, n, seed):
    """Random weights of format t with sane scales (quant bytes random, fp16 scales ~1e-2)."""
    rng = np.random.default_rng(seed)
    if t in (1, 30):
        v = (rng.standard_normal(rows * n) * 0.05).astype(np.float32)
        if t == 1:
            return v.astype(np.float16).view(np.uint8).copy()
        return (v.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).copy()
    offs, bb, be = SCALES[t]
    raw = rng.integers(0, 256, size=rows * oracle.row_bytes(t, n), dtype=np.uint8)
    blocks = raw.reshape(-1, bb)
    for o in offs:
        sc = (rng.random(blocks.shape[0]) * 0.02 + 0.001).astype(np.float16).view(np.uint8).reshape(-1, 2)
        blocks[:, o:o + 2] = sc
    return raw


@pytest.mark.parametrize("name", list(FORMATS))
def test_dequant_matches_reference_fixture(fh3, name):
    import torch
    t, rows, cols, raw, ref = _fixture(name)
    got = fh3.dequant(t, torch.from_numpy(raw).cuda(), cols, rows).cpu().numpy()
    assert _same(got, ref)


@pytest.mark.parametrize("t", [0, 1, 30, 8, 10, 11, 13, 14])
def test_dequant_random_bytes_bitexact_vs_oracle(fh3, oracle, t):
    import torch
    rows, n = 5, 768
    raw = np.random.default_rng(t).integers(0, 256, size=rows * oracle.row_bytes(t, n), dtype=np.uint8)
    got = fh3.dequant(t, torch.from_numpy(raw).cuda(), n, rows).cpu().numpy()
    assert _same(got, oracle.dequant(t, raw, rows, n))


@pytest.mark.parametrize("name", [f for f in FORMATS if f != "Q4_K"])
def test_matmul_reference_cases(fh3, golden_cases, name):
    import torch
    t, K, N, M = (int(v) for v in golden_cases[f"fmt_{name}/dims"])
    w = fh3.Weight.from_bytes(golden_cases[f"fmt_{name}/w"], K, N, type_=t)
    x = torch.from_numpy(golden_cases[f"fmt_{name}/x"]).cuda()
    b = torch.from_numpy(golden_cases[f"fmt_{name}/bias"]).cuda()
    got = fh3.matmul(w, x, b).cpu().numpy()
    assert rel_fro(got, golden_cases[f"fmt_{name}/y"]) <= TOL
    host = fh3.matmul_host(golden_cases[f"fmt_{name}/w"], K, N, golden_cases[f"fmt_{name}/x"],
                           golden_cases[f"fmt_{name}/bias"], type_=t)
    assert rel_fro(host, golden_cases[f"fmt_{name}/y"]) <= TOL


@pytest.mark.parametrize("t", [0, 1, 30, 8, 10, 11, 13, 14])
@pytest.mark.parametrize("M", [1, 5, 40])
def test_matmul_vs_oracle(fh3, oracle, t, M):
    import torch
    K, N = 1024, 300
    raw = (np.random.default_rng(t).standard_normal(N * K).astype(np.float32) * 0.05).view(np.uint8) \
        if t == 0 else _weights(oracle, t, N, K, seed=t + 100)
    x = oracle.rng_normal(t + 7, M, M * K).reshape(M, K)
    bias = oracle.rng_normal(t + 7, 99, N)
    ref = oracle.matmul(t, raw, K, N, x, bias)
    w = fh3.Weight.from_bytes(raw, K, N, type_=t)
    got = fh3.matmul(w, torch.from_numpy(x).cuda(), torch.from_numpy(bias).cuda()).cpu().numpy()
    assert rel_fro(got, ref) <= TOL


@pytest.mark.parametrize("M", [3, 40])
def test_matmul_in_row_chunks(fh3, oracle, M):
    """8200 x 8192 Q6_K: 3 tokens on the GEMV; 40 tokens through the split-bf16 GEMM, whose
    537 MB of expanded weight rows are processed in three chunks of whole 256-row tiles."""
    import torch
    t, K, N = 14, 8192, 8200
    raw = _weights(oracle, t, N, K, seed=5)
    x = oracle.rng_normal(5, 1, M * K).reshape(M, K)
    ref = oracle.matmul(t, raw, K, N, x)
    got = fh3.matmul(fh3.Weight.from_bytes(raw, K, N, type_=t), torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_fro(got, ref) <= TOL


@pytest.mark.parametrize("t", [0, 1, 13])
def test_matmul_odd_widths_and_many_tokens(fh3, oracle, t):
    """A width that is not a multiple of 16 (padded with zeros in the split operands) for the
    element formats, and more tokens than one 256-row tile."""
    import torch
    K = 1000 if t in (0, 1) else 1280
    N, M = 333, 700
    raw = (np.random.default_rng(t).standard_normal(N * K).astype(np.float32) * 0.05).view(np.uint8) \
        if t == 0 else _weights(oracle, t, N, K, seed=t + 200)
    x = oracle.rng_normal(t + 9, M, M * K).reshape(M, K)
    bias = oracle.rng_normal(t + 9, 98, N)
    ref = oracle.matmul(t, raw, K, N, x, bias)
    w = fh3.Weight.from_bytes(raw, K, N, type_=t)
    got = fh3.matmul(w, torch.from_numpy(x).cuda(), torch.from_numpy(bias).cuda()).cpu().numpy()
    assert rel_fro(got, ref) <= TOL


def test_rejects_formats_without_dequantiser_and_partial_blocks(fh3):
    import torch
    x = torch.zeros((2, 512), device="cuda")
    data = torch.zeros(4 * 512 * 2, dtype=torch.uint8, device="cuda")
    with pytest.raises(fh3.Fh3CudaError):
        fh3.matmul(fh3.Weight(data, 512, 4, 2), x)          # Q4_0: fh3_dequant has no expander
    with pytest.raises(fh3.Fh3CudaError):
        fh3.matmul(fh3.Weight(data, 300, 4, 13), x[:, :300])  # Q5_K with a partial block
