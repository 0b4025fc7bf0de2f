"""Q4_K -> fp32 on the GPU must be bit-exact with fh3_dequant (src/core/fh3_quant.c:154-196)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import read_q4k_golden

pytestmark = pytest.mark.gpu
Q4K = 12


def _gpu_dequant(fh3, raw: np.ndarray, rows: int, n: int) -> np.ndarray:
    import torch
    src = torch.from_numpy(np.ascontiguousarray(raw)).cuda()
    out = torch.full((rows, n), -7.0, dtype=torch.float32, device="cuda")
    fh3.dequant(Q4K, src, n, rows, out=out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_reference_golden_bitexact(fh3):
    t, rows, cols, raw, ref = read_q4k_golden()
    got = _gpu_dequant(fh3, raw, rows, cols)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_reference_generated_case_bitexact(fh3, golden_cases):
    got = _gpu_dequant(fh3, golden_cases["dequant/w"], 3, 1024)
    assert np.array_equal(got.view(np.uint32), golden_cases["dequant/y"].view(np.uint32))


@pytest.mark.parametrize("rows,n", [(1, 256), (37, 5120), (300, 13824)])
def test_random_bytes_bitexact_vs_oracle(fh3, oracle, rows, n):
    # Arbitrary bytes exercise every scale/min bit pattern, incl. fp16 subnormal, inf and
    # NaN d/dmin.  Every non-NaN output is bit-exact; where the reference yields NaN the GPU
    # yields NaN too, but not the same payload (x86 propagates the input NaN's payload, the
    # GPU returns the canonical NaN), so NaNs are compared as NaNs.
    rng = np.random.default_rng(rows * 7 + n)
    raw = rng.integers(0, 256, size=rows * oracle.row_bytes(Q4K, n), dtype=np.uint8)
    got = _gpu_dequant(fh3, raw, rows, n)
    ref = oracle.dequant_rows(raw, rows, n)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    # with finite scales (what real Q4_K files hold) every output is bit-exact, NaN-free
    blocks = raw.reshape(-1, 144).copy()
    blocks[:, 0:2] = np.frombuffer(np.float16(0.0123).tobytes(), np.uint8)
    blocks[:, 2:4] = np.frombuffer(np.float16(0.0456).tobytes(), np.uint8)
    raw2 = blocks.reshape(-1)
    got2 = _gpu_dequant(fh3, raw2, rows, n)
    ref2 = oracle.dequant_rows(raw2, rows, n)
    assert not np.isnan(ref2).any()
    assert np.array_equal(got2.view(np.uint32), ref2.view(np.uint32))


def test_partial_trailing_block_is_left_untouched(fh3, oracle):
    # fh3_dequant writes n/256 whole blocks only (src/core/fh3_quant.c:155)
    n = 300
    raw = oracle.make_weights(seed=1, stream=2, rows=2, n=512)[: 2 * 288]
    got = _gpu_dequant(fh3, raw, 2, n)
    ref0 = oracle.dequant_q4k(raw[:288], 256)
    assert np.array_equal(got[0, :256].view(np.uint32), ref0.view(np.uint32))
    assert np.all(got[:, 256:] == -7.0)


def test_rejects_bad_arguments(fh3):
    import torch
    buf = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    out = torch.zeros(256, dtype=torch.float32, device="cuda")
    with pytest.raises(fh3.Fh3CudaError) as e:
        fh3.dequant(2, buf, 256, 1, out=out)    # Q4_0: fh3_dequant has no expander for it
    assert e.value.code == -8
    with pytest.raises(fh3.Fh3CudaError):
        fh3.dequant(Q4K, buf[1:], 256, 1, out=out)  # misaligned source
