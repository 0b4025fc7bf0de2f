"""The elementwise ops around the GEMMs, and the weight generator, on the GPU."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu


def test_to_bf16_is_round_to_nearest_even(fh3):
    import torch
    x = torch.randn(10_001, device="cuda") * 3.0
    assert torch.equal(fh3.to_bf16(x), x.to(torch.bfloat16))


def test_rmsnorm_modulate_vs_oracle(fh3, oracle):
    import torch
    n, dim = 9, 5120
    x = oracle.rng_normal(1, 1, n * dim).reshape(n, dim)
    nw = oracle.rng_normal(1, 2, dim)
    sh = 0.1 * oracle.rng_normal(1, 3, dim)
    sc = 0.1 * oracle.rng_normal(1, 4, dim)
    ref = oracle.modulate(oracle.rmsnorm(x, nw, 1e-6), np.tile(sh, (n, 1)), np.tile(sc, (n, 1)))
    got = fh3.rmsnorm_modulate(torch.from_numpy(x).cuda(), torch.from_numpy(sh).cuda(),
                               torch.from_numpy(sc).cuda(), norm_w=torch.from_numpy(nw).cuda(), eps=1e-6)
    # output is bf16 (the GEMM operand): half an ulp of bf16
    assert rel_fro(got.float().cpu().numpy(), ref) <= 4e-3
    assert np.abs(got.float().cpu().numpy() - ref).max() <= np.abs(ref).max() * 2 ** -8


@pytest.mark.parametrize("n,dim", [(5, 512), (4, 1000), (3, 8192), (3, 10000), (4, 5121), (300, 5120)])
def test_rmsnorm_modulate_every_row_width(fh3, oracle, n, dim):
    """Both kernels: rows of up to 8 x 1024 float4 held in registers (one HBM read), and the
    general one (widths not a multiple of 4, or wider)."""
    import torch
    x = oracle.rng_normal(2, 1, n * dim).reshape(n, dim) * 3.0
    nw = oracle.rng_normal(2, 2, dim)
    sh = 0.1 * oracle.rng_normal(2, 3, dim)
    sc = 0.1 * oracle.rng_normal(2, 4, dim)
    for w in (nw, None):
        r = oracle.rmsnorm(x, w if w is not None else np.ones(dim, np.float32), 1e-6)
        ref = oracle.modulate(r, np.tile(sh, (n, 1)), np.tile(sc, (n, 1)))
        got = fh3.rmsnorm_modulate(torch.from_numpy(x).cuda(), torch.from_numpy(sh).cuda(),
                                   torch.from_numpy(sc).cuda(), norm_w=None if w is None else torch.from_numpy(w).cuda(),
                                   eps=1e-6).float().cpu().numpy()
        assert np.abs(got - ref).max() <= np.abs(ref).max() * 2 ** -8, (n, dim)


def test_swiglu_vs_reference_golden(fh3, golden_cases):
    import torch
    h = golden_cases["swiglu/h"]
    got = fh3.swiglu(torch.from_numpy(h).cuda()).cpu().numpy()
    ref = golden_cases["swiglu/y"]
    assert got[0, 0] == 0.0 and got[0, 1] == 0.0
    assert rel_fro(got, ref) <= 1e-6


def test_device_weight_generator_statistics(fh3, oracle):
    import torch
    rows, n = 512, 5120
    w = fh3.make_weights(rows, n, seed=0, stream_id=11, scale=0.02)
    wf = fh3.dequant(12, w.data, n, rows).cpu().numpy()
    assert abs(wf.std() - 0.02) < 0.002 and abs(wf.mean()) < 1e-3
    # round trip: the same blocks re-quantised on the CPU from the dequantised values are close
    raw_cpu = oracle.quantize_q4k(wf[:8])
    assert rel_fro(oracle.dequant_rows(raw_cpu, 8, n), wf[:8]) < 0.12
    # deterministic
    w2 = fh3.make_weights(rows, n, seed=0, stream_id=11, scale=0.02)
    assert torch.equal(w.data, w2.data)
