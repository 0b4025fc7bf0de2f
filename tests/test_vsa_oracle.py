"""The VSA oracle (oracle/fh3_oracle.c: oracle_vsa) pinned to the reference.

fh3_vsa_attention (src/core/fh3_vsa.c:186-507) is checked by the reference's
tests/unit/test_vsa.c against three fixtures at rel-L2 <= 1e-5; the oracle meets
the same bar on the same files, equals the reference's own compiled function bit
for bit on the reference-computed cases in ref_cases.npz (ties, no gate, prefix
tiles of 32 and 100, both geometry fallbacks), and with sparsity 0 and no gate it
is dense attention (test_vsa.c:266-274).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import VSA_CASES, VSA_FIXTURES, read_vsa_golden, rel_l2, vsa_case


@pytest.mark.parametrize("name", VSA_FIXTURES)
def test_vsa_oracle_matches_reference_fixture(oracle, name):
    seq, heads, hd, sp, q, k, v, gate, ref = read_vsa_golden(name)
    out = oracle.vsa(q, k, v, gate, seq, heads, hd, 64, sp)
    assert rel_l2(out, ref) <= 1e-5


@pytest.mark.parametrize("name", VSA_CASES)
def test_vsa_oracle_bitwise_equals_reference_case(oracle, golden_cases, name):
    seq, heads, hd, tile, sp, q, k, v, gate, y = vsa_case(golden_cases, name)
    out = oracle.vsa(q, k, v, gate, seq, heads, hd, tile, sp)
    np.testing.assert_array_equal(out, y)


def test_vsa_oracle_sparsity0_without_gate_is_dense_attention(oracle):
    seq, heads, hd, _, q, k, v, _, _ = read_vsa_golden("vsa_sparsity0")
    fine = oracle.vsa(q, k, v, None, seq, heads, hd, 64, 0.0)
    dense = oracle.attention(q, k, v, heads, hd)
    assert rel_l2(fine, dense) <= 1e-5


def test_vsa_oracle_geometry():
    """Tile counts of build_vsa_geometry (src/core/fh3_vsa.c:32-161) on the fixture shapes."""
    from oracle.oracle import Oracle
    o = Oracle()
    assert o.vsa_tiles((784, 0, 0, 784, 7, 8, 14)) == (16, 0, 16)       # 2 x 2 x 4 cells
    assert o.vsa_tiles((268, 35, 23, 210, 5, 6, 7)) == (10, 2, 8)       # 1 text + 1 audio, 2 x 2 x 2
    assert o.vsa_tiles((258, 130, 0, 128, 4, 4, 8), tile=100) == (4, 2, 2)
    assert o.vsa_tiles((200, 50, 50, 50, 2, 5, 5)) == (50, 0, 50)       # counts mismatch: all video, grid 1x1x200
    assert o.vsa_tiles((170, 20, 0, 150, 3, 7, 7)) == (39, 1, 38)      # grid mismatch: 1 x 1 x 150


def test_vsa_oracle_ties_keep_lowest_tile_index(oracle, golden_cases):
    """With every video key tile scoring the same, the kept ones are the first k (cmp_tile_score)."""
    seq, heads, hd, tile, sp, q, k, v, gate, _ = vsa_case(golden_cases, "hd128_tied")
    _, sc, mk = oracle.vsa(q, k, v, gate, seq, heads, hd, tile, sp, want_tiles=True)
    nt, npre, nvid = oracle.vsa_tiles(seq, tile)
    kv = int(np.ceil(np.float32(1.0 - np.float32(sp)) * np.float32(nvid)))
    for h in range(heads):
        for i in range(npre, nt):
            assert np.all(sc[h, i, npre:] == sc[h, i, npre])
            assert list(np.nonzero(mk[h, i, npre:])[0]) == list(range(kv))
