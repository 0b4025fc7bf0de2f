"""The CPU oracle, pinned against the reference's golden vectors and the reference itself.

Mirrors the reference's own checks: tests/unit/test_quant.c (dequant bit-exact vs
gguf-py) and tests/unit/test_matmul.c (matmul rel-L2 <= 1e-6 vs fp64 numpy), plus
bitwise equality with fh3_matmul (whose scalar/AVX2/OpenMP variants agree bitwise,
test_matmul.c:107-139) on the reference-generated cases in tests/golden/ref_cases.npz.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import (close_like_reference, read_matmul_golden, read_q4k_golden, read_rmsnorm_golden,
                      read_rope3_golden, rel_fro)

Q4K = 12


def test_dequant_matches_reference_golden_bitexact(oracle):
    t, rows, cols, raw, ref = read_q4k_golden()
    assert (t, rows, cols) == (12, 4, 512)
    got = oracle.dequant_rows(raw, rows, cols)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_matmul_matches_reference_golden(oracle):
    t, K, N, M, w, x, bias, y = read_matmul_golden()
    assert (t, K, N, M) == (12, 5376, 192, 37)
    got = oracle.matmul(Q4K, w, K, N, x, bias)
    # tests/unit/test_matmul.c:287-300: rel-L2 vs the fp64 reference <= 1e-6
    assert rel_fro(got, y) <= 1e-6


def test_matmul_bitwise_equals_reference_cases(oracle, golden_cases):
    names = sorted({k.split("/")[0] for k in golden_cases if k.startswith("k")})
    assert len(names) >= 6
    for name in names:
        K, N, M = (int(v) for v in golden_cases[f"{name}/dims"])
        bias = golden_cases.get(f"{name}/bias")
        got = oracle.matmul(Q4K, golden_cases[f"{name}/w"], K, N, golden_cases[f"{name}/x"], bias)
        ref = golden_cases[f"{name}/y"]
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), name


def test_dequant_and_swiglu_bitwise_equal_reference_cases(oracle, golden_cases):
    got = oracle.dequant_rows(golden_cases["dequant/w"], 3, 1024)
    assert np.array_equal(got.view(np.uint32), golden_cases["dequant/y"].view(np.uint32))
    sw = oracle.swiglu(golden_cases["swiglu/h"])
    assert np.array_equal(sw.view(np.uint32), golden_cases["swiglu/y"].view(np.uint32))
    assert sw[0, 0] == 0.0 and sw[0, 1] == 0.0  # gates -100 and -80.5: the g < -80 cut


def test_rng_matches_reference_fh3_rng_normal(oracle, golden_cases):
    got = oracle.rng_normal(7, 3, 1001)
    assert np.array_equal(got.view(np.uint32), golden_cases["rng/seed7_stream3"].view(np.uint32))


def test_oracle_bitwise_equals_live_reference(oracle, reference):
    rng = np.random.default_rng(5)
    for K, N, M in [(256, 3, 2), (512, 65, 9), (1280, 129, 33), (5120, 64, 3)]:
        w = oracle.make_weights(seed=int(rng.integers(1 << 30)), stream=1, rows=N, n=K)
        x = oracle.rng_normal(int(rng.integers(1 << 30)), 2, M * K).reshape(M, K)
        b = oracle.rng_normal(3, 4, N)
        for bias in (None, b):
            a = oracle.matmul(Q4K, w, K, N, x, bias)
            r = reference.matmul(Q4K, w, K, N, x, bias)
            assert np.array_equal(a.view(np.uint32), r.view(np.uint32)), (K, N, M)
    x = oracle.rng_normal(1, 3, 8 * 5120).reshape(8, 5120)
    nw = oracle.rng_normal(1, 4, 5120)
    sh = oracle.rng_normal(1, 5, 8 * 5120).reshape(8, 5120)
    sc = oracle.rng_normal(1, 6, 8 * 5120).reshape(8, 5120)
    for a, r in [(oracle.rmsnorm(x, nw, 1e-6), reference.rmsnorm(x, nw, 1e-6)),
                 (oracle.modulate(x, sh, sc), reference.modulate(x, sh, sc)),
                 (oracle.gate_residual(x, sh, sc), reference.gate_residual(x, sh, sc))]:
        assert np.array_equal(a.view(np.uint32), r.view(np.uint32))


def _subblock_bound(raw: np.ndarray, rows: int, n: int, oracle) -> np.ndarray:
    """Per-weight round-trip bound of the quantiser: dl/2 + 7.5 d + dmin/2 (+ fp32 slack)."""
    blocks = raw.reshape(rows * n // 256, 144)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dmin = blocks[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    s = blocks[:, 4:16].astype(np.int32)
    sc = np.zeros((blocks.shape[0], 8), np.float32)
    for j in range(8):
        if j < 4:
            sc[:, j] = s[:, j] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 15) | ((s[:, j - 4] >> 6) << 4)
    dl = d[:, None] * sc
    bound = 0.5 * dl + 7.5 * d[:, None] + 0.5 * dmin[:, None] + 1e-6
    return np.repeat(bound, 32, axis=1).reshape(rows, n)


@pytest.mark.parametrize("scale", [0.02, 1.0, 37.0])
def test_quantiser_round_trip_bounds(oracle, scale):
    rows, n = 16, 1024
    x = (scale * oracle.rng_normal(11, 12, rows * n)).reshape(rows, n)
    raw = oracle.quantize_q4k(x)
    dq = oracle.dequant_rows(raw, rows, n)
    err = np.abs(dq - x)
    assert np.all(err <= _subblock_bound(raw, rows, n, oracle))
    assert rel_fro(dq, x) < 0.12  # 4.5-bit quantisation of a normal


def test_quantiser_edge_blocks(oracle):
    n = 256
    cases = [np.zeros(n), np.full(n, 0.5), np.full(n, -0.25), np.linspace(0.0, 1.0, n),
             np.linspace(-2.0, -1.0, n), np.where(np.arange(n) % 2 == 0, 3.0, -3.0)]
    x = np.stack(cases).astype(np.float32)
    raw = oracle.quantize_q4k(x)
    dq = oracle.dequant_rows(raw, x.shape[0], n)
    assert np.all(np.abs(dq - x) <= _subblock_bound(raw, x.shape[0], n, oracle))
    assert np.all(dq[0] == 0.0)


def test_make_weights_equals_quantise_of_rng(oracle):
    w = oracle.make_weights(seed=3, stream=9, rows=5, n=512, scale=0.02)
    x = 0.02 * oracle.rng_normal(3, 9, 5 * 512)
    assert np.array_equal(w, oracle.quantize_q4k(x.reshape(5, 512)))


def test_oracle_rejects_bad_arguments(oracle):
    with pytest.raises(ValueError):
        oracle.matmul(99, np.zeros(144, np.uint8), 256, 1, np.zeros((1, 256), np.float32))
    with pytest.raises(ValueError):
        oracle.quantize_q4k(np.zeros((1, 100), np.float32))


def test_rmsnorm_matches_reference_op_fixture(oracle):
    """tests/fixtures/ops/rmsnorm.bin of the reference, with its own tolerance rule."""
    n, dim, eps, x, w, ref = read_rmsnorm_golden()
    assert close_like_reference(oracle.rmsnorm(x, w, eps), ref)


def test_rope3_matches_reference_op_fixture(oracle):
    """tests/fixtures/ops/rope3.bin (rot_dim 96 of head_dim 128), with the reference's tolerance."""
    n, heads, hd, rot, x, c, s, ref = read_rope3_golden()
    got = oracle.rope3(x, c, s, heads, hd, rot)
    assert close_like_reference(got, ref)
    # channels past rot_dim are untouched
    xv, gv = x.reshape(n, heads, hd), got.reshape(n, heads, hd)
    assert np.array_equal(xv[:, :, rot:], gv[:, :, rot:])


def test_qk_norm_rope_bitwise_equals_reference_case(oracle, golden_cases):
    """fh3_dit.c:397-401 (per-head rmsnorm, then rope3) computed by the reference itself."""
    n, H, D, R = (int(v) for v in golden_cases["qkrope/dims"])
    got = oracle.qk_norm_rope(golden_cases["qkrope/x"], golden_cases["qkrope/w"], golden_cases["qkrope/cos"],
                              golden_cases["qkrope/sin"], H, D, R, 1e-6)
    assert np.array_equal(got.view(np.uint32), golden_cases["qkrope/y"].view(np.uint32))


def test_rope3_bitwise_equals_live_reference(oracle, reference):
    rng = np.random.default_rng(3)
    for n, H, D, R in ((3, 2, 128, 96), (2, 3, 64, 64), (1, 1, 16, 2)):
        x = rng.standard_normal((n, H * D)).astype(np.float32)
        c = rng.standard_normal((n, R)).astype(np.float32)
        s = rng.standard_normal((n, R)).astype(np.float32)
        a, b = oracle.rope3(x, c, s, H, D, R), reference.rope3(x, c, s, H, D, R)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (n, H, D, R)


def test_attention_bitwise_equals_reference_case(oracle, golden_cases):
    """fh3_attention on n = 200 (a partial 64-key tile), 2 heads x 128, computed by the reference."""
    n, H, D = (int(v) for v in golden_cases["attn/dims"])
    got = oracle.attention(golden_cases["attn/q"], golden_cases["attn/k"], golden_cases["attn/v"], H, D)
    assert np.array_equal(got.view(np.uint32), golden_cases["attn/y"].view(np.uint32))


def test_attention_matches_reference_op_fixture(oracle):
    """The reference's tests/fixtures/ops/attention.bin (n = 777, 4 heads x 128; 6.4 MB, read in
    place where the reference tree exists, not copied), with its own tolerance rule."""
    import os
    import struct
    from oracle.oracle import REF_TREE
    path = os.path.join(REF_TREE, "tests", "fixtures", "ops", "attention.bin") if REF_TREE else ""
    if not path or not os.path.exists(path):
        pytest.skip("reference tree not present")
    with open(path, "rb") as f:
        b = f.read()
    n, heads, hd = struct.unpack("<III", b[:12])
    a = np.frombuffer(b[12:], np.float32)
    c = n * heads * hd
    q, k, v, ref = (a[i * c:(i + 1) * c].reshape(n, heads * hd) for i in range(4))
    assert close_like_reference(oracle.attention(q, k, v, heads, hd), ref)


FORMATS = ("F16", "BF16", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K")


def _read_format_golden(name):
    import os
    import struct
    from conftest import GOLDEN
    with open(os.path.join(GOLDEN, f"{name}.bin"), "rb") as f:
        b = f.read()
    t, rows, cols, nb = struct.unpack("<IIII", b[:16])
    raw = np.frombuffer(b[16:16 + nb], np.uint8).copy()
    ref = np.frombuffer(b[16 + nb:], np.float32).reshape(rows, cols).copy()
    return t, rows, cols, raw, ref


@pytest.mark.parametrize("name", FORMATS)
def test_dequant_formats_match_reference_goldens(oracle, name):
    """tests/fixtures/quant/<format>.bin of the reference (gguf-py 0.19.0 output): bit-exact."""
    t, rows, cols, raw, ref = _read_format_golden(name)
    got = oracle.dequant(t, raw, rows, cols)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("name", [f for f in FORMATS if f != "Q4_K"])
def test_matmul_formats_bitwise_equal_reference_cases(oracle, golden_cases, name):
    t, K, N, M = (int(v) for v in golden_cases[f"fmt_{name}/dims"])
    got = oracle.matmul(t, golden_cases[f"fmt_{name}/w"], K, N, golden_cases[f"fmt_{name}/x"],
                        golden_cases[f"fmt_{name}/bias"])
    assert np.array_equal(got.view(np.uint32), golden_cases[f"fmt_{name}/y"].view(np.uint32))


def test_dequant_formats_bitwise_equal_live_reference_on_random_blocks(oracle, reference):
    rng = np.random.default_rng(11)
    for t in (1, 30, 8, 10, 11, 12, 13, 14):
        n = 768
        rb = oracle.row_bytes(t, n)
        raw = rng.integers(0, 256, size=rb * 2, dtype=np.uint8)
        got = oracle.dequant(t, raw, 2, n)
        live = np.stack([reference.dequant(t, raw[i * rb:(i + 1) * rb], n) for i in range(2)])
        nan = np.isnan(got)
        assert np.array_equal(nan, np.isnan(live)), t
        assert np.array_equal(got[~nan].view(np.uint32), live[~nan].view(np.uint32)), t
