"""Video sparse attention (fh3_vsa_attention, src/core/fh3_vsa.c:186-507) on the GPU.

Three bars:
* the tile stage (tile means, tile scores, kept key tiles) is computed in fp32 in the
  reference's order, so the scores and the 0/1 tile mask equal the oracle's BIT FOR BIT
  (the oracle equals the reference's compiled function, tests/test_vsa_oracle.py);
* fp32 operands run the fine pass in fp32: the output meets the reference's own bar,
  relative L2 error <= 1e-5 against its fixtures (tests/unit/test_vsa.c:175);
* bf16 operands run it on tensor cores with fp32 softmax and accumulation: relative L2
  (Frobenius) error <= 1e-2 against fp32 attention on the same bf16-rounded inputs.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import VSA_CASES, VSA_FIXTURES, read_vsa_golden, rel_l2, vsa_case

pytestmark = pytest.mark.gpu
TOL = 1e-2      # bf16 operands
TOL_F32 = 1e-5  # fp32 operands, the reference's bar


@pytest.fixture(autouse=True, params=["tc", "mma"])
def vsa_kernel(request, monkeypatch):
    """bf16 head_dim-128 cases on both fine passes: tcgen05 with an M = 64 query tile
    (tile-order operands, TMEM tiles; the default for tiles of at most 64 tokens) and
    mma.sync (FH3CUDA_VSA_KERNEL=mma; the default for head_dim 64 and for larger tiles)."""
    if request.param == "mma":
        monkeypatch.setenv("FH3CUDA_VSA_KERNEL", request.param)
    else:
        monkeypatch.delenv("FH3CUDA_VSA_KERNEL", raising=False)
    return request.param


def _dev(a, bf16=False):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    return t.to(torch.bfloat16) if bf16 else t


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("name", VSA_FIXTURES)
def test_tile_mask_bitwise_equals_oracle_on_fixture(fh3, oracle, name):
    seq, heads, hd, sp, q, k, v, gate, _ = read_vsa_golden(name)
    _, sc_ref, mk_ref = oracle.vsa(q, k, v, gate, seq, heads, hd, 64, sp, want_tiles=True)
    sc, mk = fh3.vsa_tiles(_dev(q), _dev(k), seq, heads, hd, 64, sp)
    np.testing.assert_array_equal(sc.cpu().numpy(), sc_ref)
    np.testing.assert_array_equal(mk.cpu().numpy(), mk_ref)


@pytest.mark.parametrize("name", VSA_FIXTURES)
def test_fp32_output_matches_reference_fixture(fh3, name):
    seq, heads, hd, sp, q, k, v, gate, ref = read_vsa_golden(name)
    got = _np(fh3.vsa_attention(_dev(q), _dev(k), _dev(v), None if gate is None else _dev(gate), seq, heads, hd,
                                64, sp))
    assert rel_l2(got, ref) <= TOL_F32


@pytest.mark.parametrize("name", VSA_FIXTURES)
def test_bf16_output_vs_oracle_on_fixture(fh3, oracle, name):
    """The fixture's q/k/v/gate rounded to bf16: tensor-core fine pass against fp32 VSA on the
    same rounded values; the mask must still be the oracle's."""
    seq, heads, hd, sp, q, k, v, gate, _ = read_vsa_golden(name)
    qb, kb, vb, gb = (_dev(a, True) for a in (q, k, v, gate))
    got = _np(fh3.vsa_attention(qb, kb, vb, gb, seq, heads, hd, 64, sp))
    same, sc_ref, mk_ref = oracle.vsa(_np(qb), _np(kb), _np(vb), _np(gb), seq, heads, hd, 64, sp, want_tiles=True)
    sc, mk = fh3.vsa_tiles(qb, kb, seq, heads, hd, 64, sp)
    np.testing.assert_array_equal(sc.cpu().numpy(), sc_ref)
    np.testing.assert_array_equal(mk.cpu().numpy(), mk_ref)
    assert rel_l2(got, same) <= TOL


@pytest.mark.parametrize("name", VSA_CASES)
def test_reference_cases(fh3, oracle, golden_cases, name):
    """Ties, no gate, prefix tiles of 32 and of 100 tokens (two 64-row CTAs a tile), both
    geometry fallbacks; the reference computed y (ref_cases.npz)."""
    seq, heads, hd, tile, sp, q, k, v, gate, y = vsa_case(golden_cases, name)
    _, sc_ref, mk_ref = oracle.vsa(q, k, v, gate, seq, heads, hd, tile, sp, want_tiles=True)
    sc, mk = fh3.vsa_tiles(_dev(q), _dev(k), seq, heads, hd, tile, sp)
    np.testing.assert_array_equal(sc.cpu().numpy(), sc_ref)
    np.testing.assert_array_equal(mk.cpu().numpy(), mk_ref)
    got = _np(fh3.vsa_attention(_dev(q), _dev(k), _dev(v), None if gate is None else _dev(gate), seq, heads, hd,
                                tile, sp))
    assert rel_l2(got, y) <= TOL_F32


@pytest.mark.parametrize("hd,out_bf16", [(128, False), (128, True), (64, True)])
def test_bf16_inputs_strided_views(fh3, oracle, hd, out_bf16):
    """bf16 q/k/v/gate as the thirds of one [n][3*heads*hd] buffer (a QKV output) and a
    gate with padded rows; the mask must still equal the oracle's on the same values."""
    import torch
    seq = (24 + 40 + 4 * 8 * 12, 24, 40, 384, 4, 8, 12)
    n, heads = seq[0], 3
    w = heads * hd
    g = torch.Generator(device="cuda").manual_seed(hd)
    qkv = torch.randn((n, 3 * w), device="cuda", generator=g).to(torch.bfloat16)
    gate = torch.randn((n, w + 8), device="cuda", generator=g).to(torch.bfloat16)[:, :w]
    q, k, v = qkv[:, :w], qkv[:, w:2 * w], qkv[:, 2 * w:]
    got = _np(fh3.vsa_attention(q, k, v, gate, seq, heads, hd, 64, 0.75, out_bf16=out_bf16))
    f = lambda t: np.ascontiguousarray(_np(t))
    ref, sc_ref, mk_ref = oracle.vsa(f(q), f(k), f(v), f(gate), seq, heads, hd, 64, 0.75, want_tiles=True)
    sc, mk = fh3.vsa_tiles(q, k, seq, heads, hd, 64, 0.75)
    np.testing.assert_array_equal(sc.cpu().numpy(), sc_ref)
    np.testing.assert_array_equal(mk.cpu().numpy(), mk_ref)
    assert rel_l2(got, ref) <= TOL


def test_sparsity0_without_gate_equals_dense_attention(fh3):
    """The reference's structural check (tests/unit/test_vsa.c:266-274) on the GPU: at sparsity 0
    and no gate every key tile is kept, so VSA is the dense attention kernel up to summation order."""
    import torch
    seq = (100 + 4 * 8 * 8, 100, 0, 256, 4, 8, 8)
    n, heads = seq[0], 2
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn((n, heads * 128), device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    got = _np(fh3.vsa_attention(q, k, v, None, seq, heads, 128, 64, 0.0))
    dense = _np(fh3.attention(q, k, v, heads))
    assert rel_l2(got, dense) <= 5e-3


def test_model_sized_sequence_properties(fh3, oracle):
    """A bench-shaped sequence (audio prefix + 21 x 30 x 52 video grid, 40 heads x 128): every
    video query row keeps exactly npre + k tiles, prefix rows keep all, and the GPU's kept tiles
    of a sample of rows equal the oracle's ranking of the GPU's own (bit-exact) scores."""
    import torch
    seq = (1024 + 21 * 30 * 52, 0, 1024, 21 * 30 * 52, 21, 30, 52)
    n, heads, hd, sp = seq[0], 40, 128, 0.8
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k = (torch.randn((n, heads * hd), device="cuda", generator=g).to(torch.bfloat16) for _ in range(2))
    nt, npre, nvid = fh3.vsa_num_tiles(seq)
    assert (nt, npre, nvid) == (640, 16, 624)
    sc, mk = fh3.vsa_tiles(q, k, seq, heads, hd, 64, sp)
    kv = int(np.ceil(np.float32(1.0 - np.float32(sp)) * np.float32(nvid)))
    cnt = mk.sum(dim=2).cpu().numpy()
    assert np.all(cnt[:, :npre] == nt) and np.all(cnt[:, npre:] == npre + kv)
    s = sc.cpu().numpy()
    m = mk.cpu().numpy()
    for h, i in ((0, npre), (7, 300), (39, nt - 1)):
        row = s[h, i, npre:]
        order = sorted(range(nvid), key=lambda j: (-row[j], j))
        want = np.zeros(nvid, np.uint8)
        want[order[:kv]] = 1
        np.testing.assert_array_equal(m[h, i, npre:], want)


def test_rejects_bad_arguments(fh3):
    import torch
    from fasth3inc_b200 import Fh3CudaError
    seq = (64, 0, 0, 64, 4, 4, 4)
    x = torch.zeros((64, 96), device="cuda")
    with pytest.raises(Fh3CudaError):
        fh3.vsa_attention(x, x, x, None, seq, 1, 96)           # head_dim 96
    with pytest.raises(Fh3CudaError):
        fh3.vsa_attention(x, x, x, None, (0, 0, 0, 0, 1, 1, 1), 1, 64)   # empty sequence
    xb = torch.zeros((64, 64), device="cuda", dtype=torch.bfloat16)
    y = torch.zeros((64, 130), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(Fh3CudaError):
        fh3.vsa_attention(xb, xb, xb, None, seq, 1, 64, out=y[:, 1:65])   # bf16: o not 16-byte aligned
    x64 = torch.zeros((64, 64), device="cuda")
    with pytest.raises(Fh3CudaError):
        fh3.vsa_attention(x64, x64, x64, None, seq, 1, 64, out=y[:, :64])  # fp32 operands need an fp32 o


@pytest.mark.parametrize("seq", [(64 * 3 + 7 * 9 * 10, 64 * 3, 0, 630, 7, 9, 10),      # ragged cells of 1..4 per axis
                                 (30 + 20 + 6 * 6 * 6, 30, 20, 216, 6, 6, 6)])
def test_bf16_hd128_ragged_tiles_vs_oracle(fh3, oracle, seq):
    """Ragged video cells (counts 1..64), partial prefix tiles, gate and bf16 output on head_dim 128:
    the tcgen05 pass pads every tile's run to 8 rows and masks the rest."""
    import torch
    n, heads, hd = seq[0], 2, 128
    g = torch.Generator(device="cuda").manual_seed(n)
    q, k, v, gate = (torch.randn((n, heads * hd), device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    got = _np(fh3.vsa_attention(q, k, v, gate, seq, heads, hd, 64, 0.7, out_bf16=True))
    f = lambda t: np.ascontiguousarray(_np(t))
    ref = oracle.vsa(f(q), f(k), f(v), f(gate), seq, heads, hd, 64, 0.7)
    assert rel_l2(got, ref) <= TOL
