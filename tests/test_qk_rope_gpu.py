"""q / k normalisation + rope after the QKV projection (fh3_dit.c:397-401) on the GPU:
fh3cuda_qk_norm_rope_dev against the oracle (bitwise equal to the reference's fh3_rmsnorm
then fh3_rope3, tests/test_oracle.py).  The bar is bit-exact for fp32 outputs; a bf16
output must be the fp32 result rounded once (round to nearest even)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    return t if dtype is None else t.to(dtype)


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _angles(o, seed, n, rot):
    ang = o.rng_normal(seed, 3, n * rot).reshape(n, rot)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def test_reference_case_bitexact(fh3, golden_cases):
    n, H, D, R = (int(v) for v in golden_cases["qkrope/dims"])
    got = fh3.qk_norm_rope(_t(golden_cases["qkrope/x"]), _t(golden_cases["qkrope/w"]), _t(golden_cases["qkrope/cos"]),
                           _t(golden_cases["qkrope/sin"]), H, D, R, 1e-6)
    assert np.array_equal(_bits(got.cpu().numpy()), _bits(golden_cases["qkrope/y"]))


def test_q_and_k_thirds_of_a_qkv_output(fh3, oracle):
    """The DiT shape (40 heads x 128, rot 96) read as strided views of [n][3*inner]."""
    n, H, D, R = 37, 40, 128, 96
    inner = H * D
    qkv = (oracle.rng_normal(11, 1, n * 3 * inner) * 2.0).reshape(n, 3 * inner)
    wq, wk = 1.0 + 0.1 * oracle.rng_normal(11, 2, D), 1.0 + 0.1 * oracle.rng_normal(11, 4, D)
    cs, sn = _angles(oracle, 11, n, R)
    g = _t(qkv)
    for part, w in ((0, wq), (1, wk)):
        got = fh3.qk_norm_rope(g[:, part * inner:(part + 1) * inner], _t(w), _t(cs), _t(sn), H, D, R, 1e-6)
        ref = oracle.qk_norm_rope(qkv[:, part * inner:(part + 1) * inner], w, cs, sn, H, D, R, 1e-6)
        assert np.array_equal(_bits(got.cpu().numpy()), _bits(ref)), part


def test_bf16_input_and_output(fh3, oracle):
    import torch
    n, H, D, R = 19, 8, 128, 96
    x = oracle.rng_normal(12, 1, n * H * D).reshape(n, H * D)
    w = 1.0 + 0.1 * oracle.rng_normal(12, 2, D)
    cs, sn = _angles(oracle, 12, n, R)
    xb = _t(x, torch.bfloat16)
    x_dec = xb.float().cpu().numpy()                     # the values the kernel reads
    ref = oracle.qk_norm_rope(x_dec, w, cs, sn, H, D, R, 1e-6)
    got32 = fh3.qk_norm_rope(xb, _t(w), _t(cs), _t(sn), H, D, R, 1e-6)
    assert np.array_equal(_bits(got32.cpu().numpy()), _bits(ref))
    got16 = fh3.qk_norm_rope(xb, _t(w), _t(cs), _t(sn), H, D, R, 1e-6, out_bf16=True)
    want16 = torch.from_numpy(ref).to(torch.bfloat16)
    assert torch.equal(got16.cpu().view(torch.int16), want16.view(torch.int16))


def test_in_place_and_edge_rotations(fh3, oracle):
    rng_seed = 13
    for n, H, D, R in ((5, 3, 128, 96), (4, 2, 64, 0), (3, 2, 256, 256), (2, 1, 32, 2), (9, 4, 128, 128)):
        x = oracle.rng_normal(rng_seed, 1, n * H * D).reshape(n, H * D) * 5.0
        w = 1.0 + 0.1 * oracle.rng_normal(rng_seed, 2, D)
        cs, sn = _angles(oracle, rng_seed, n, max(R, 2))
        ref = oracle.qk_norm_rope(x, w, cs[:, :R], sn[:, :R], H, D, R, 1e-5)
        buf = _t(x)
        out = fh3.qk_norm_rope(buf, _t(w), _t(cs[:, :R]) if R else None, _t(sn[:, :R]) if R else None, H, D, R,
                               1e-5, out=buf)
        assert out.data_ptr() == buf.data_ptr()
        assert np.array_equal(_bits(buf.cpu().numpy()), _bits(ref)), (n, H, D, R)
        rng_seed += 1


def test_zero_rows_and_large_values(fh3, oracle):
    n, H, D, R = 4, 2, 128, 96
    x = oracle.rng_normal(21, 1, n * H * D).reshape(n, H * D)
    x[0] = 0.0            # all-zero vector: 0 * (1 / sqrt(eps))
    x[1] *= 1.0e15        # sum of squares near the fp32 range
    x[2] *= 1.0e-20       # underflowing squares
    w = 1.0 + 0.1 * oracle.rng_normal(21, 2, D)
    cs, sn = _angles(oracle, 21, n, R)
    got = fh3.qk_norm_rope(_t(x), _t(w), _t(cs), _t(sn), H, D, R, 1e-6)
    ref = oracle.qk_norm_rope(x, w, cs, sn, H, D, R, 1e-6)
    assert np.array_equal(_bits(got.cpu().numpy()), _bits(ref))


def test_rejects_bad_arguments(fh3):
    import torch
    x = torch.zeros((2, 4 * 100), device="cuda")
    w = torch.ones(100, device="cuda")
    with pytest.raises(fh3.Fh3CudaError):
        fh3.qk_norm_rope(x, w, None, None, 4, 100, 0)          # head_dim not a multiple of 32
    x = torch.zeros((2, 256), device="cuda")
    w = torch.ones(128, device="cuda")
    cs = torch.zeros((2, 96), device="cuda")
    with pytest.raises(fh3.Fh3CudaError):
        fh3.qk_norm_rope(x, w, cs, cs, 2, 128, 95)            # odd rot_dim
    with pytest.raises(fh3.Fh3CudaError):
        fh3.qk_norm_rope(x, w, None, None, 2, 128, 96)        # rotation without cos/sin
    with pytest.raises(fh3.Fh3CudaError):
        fh3.qk_norm_rope(x[:, 1:], w, cs, cs, 1, 128, 96)     # misaligned view
