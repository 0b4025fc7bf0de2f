"""Parity at the bench's own sizes, on the bench's own path.

BASELINE config 4 (one DiT block projection set: d = 5120, 40 heads x 128, FFN 13824,
M = 16384 latent rows, cross K/V on 512 text rows of dim 5120) and config 3 (the SwiGLU
FFN: fc1 -> swiglu -> fc2 at M = 4096) run through the same launches the timed step
makes: from 2048 rows every projection takes the two-pass path (Q4_K expanded to bf16
once per call, then the TMA-fed tcgen05 pair kernel) with the rmsnorm+modulate
prologue and the bf16, SwiGLU and gated-residual epilogues; the 512-row text K/V
projection takes the fused pair kernel.

Every row is computed on the GPU; token rows are independent in every projection, so
the oracle (fh3_matmul, fh3_rmsnorm, fh3_modulate, fh3_swiglu, fh3_gate_residual
restated, src/core/fh3_ops.c:317-585) recomputes a sample of 64 rows at full width.
Two checks per sample:
  * each stage against the oracle fed the GPU's own input rows for that stage
    (relative Frobenius error <= 5e-3 per GEMM: the bf16 tensor-core bar);
  * the whole chain against the oracle composed in fp32 from the same starting rows
    (<= 1e-2 on the residual increment, <= 1e-2 on the FFN output).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu
Q4K = 12
SAMPLE = 64
GEMM_TOL = 5e-3
CHAIN_TOL = 1e-2


def _sample(n: int, k: int, seed: int) -> np.ndarray:
    """k sorted row indices of n, the first and last row included (tile edges)."""
    rng = np.random.default_rng(seed)
    mid = rng.choice(np.arange(1, n - 1), size=k - 2, replace=False)
    return np.sort(np.concatenate([[0, n - 1], mid]))


@pytest.fixture
def default_gemm_path(monkeypatch):
    monkeypatch.delenv("FH3CUDA_GEMM_KERNEL", raising=False)


def test_config4_block_projection_set_full_width(fh3, oracle, default_gemm_path):
    import torch

    from fasth3inc_b200 import _lib
    from fasth3inc_b200.trunk import Runner, Trunk, Workspace
    d, F, M, T = 5120, 13824, 16384, 512
    L = _lib.load()
    assert L.fh3cuda_gemm_launches(M) == 2          # the two-pass path, as in the timed step
    trunk = Trunk(d=d, F=F, n_blocks=1, seed=11).build()
    ws = Workspace(M, T, d=d, F=F)
    g = torch.Generator(device="cuda").manual_seed(41)
    h0 = torch.randn((M, d), device="cuda", generator=g)
    text = torch.randn((T, d), device="cuda", generator=g)
    text_bf = fh3.to_bf16(text)
    rows = _sample(M, SAMPLE, 4)
    trows = _sample(T, SAMPLE, 5)
    ri = torch.from_numpy(rows).cuda()
    ti = torch.from_numpy(trows).cuda()
    taps = {}

    def tap(stage, t):
        taps[stage] = (t.index_select(0, ti if stage == "ckv" else ri)).float().cpu().numpy()

    h = h0.clone()
    blk = trunk.blocks[0]
    Runner(trunk, ws).block(blk, h, text_bf, tap=tap)
    torch.cuda.synchronize()
    assert fh3.device_status() == 0
    assert np.isfinite(h.cpu().numpy()).all()

    raw = {k: w.data.cpu().numpy() for k, w in blk.w.items()}
    sh1, sc1, g1, shc, scc, gc, sh2, sc2, g2 = (v.cpu().numpy() for v in (
        blk.shift1, blk.scale1, blk.gate1, blk.shift_c, blk.scale_c, blk.gate_c, blk.shift2, blk.scale2,
        blk.gate2))
    n = SAMPLE
    ones = np.ones(d, np.float32)

    def norm_mod(x, shift, scale):
        return oracle.modulate(oracle.rmsnorm(x, ones, 1e-6), np.tile(shift, (n, 1)), np.tile(scale, (n, 1)))

    def mm(name, x, out, inn):
        return oracle.matmul(Q4K, raw[name], inn, out, x)

    hs = h0.cpu().numpy()[rows]
    errs = {}
    # stage by stage, each fed the GPU's own inputs
    errs["a1"] = rel_fro(taps["a1"], norm_mod(hs, sh1, sc1))
    errs["qkv"] = rel_fro(taps["qkv"], mm("qkv", taps["a1"], 3 * d, d))
    errs["o"] = rel_fro(taps["h_o"] - hs, g1 * mm("o", taps["qkv"][:, 2 * d:], d, d))
    errs["c"] = rel_fro(taps["c"], norm_mod(taps["h_o"], shc, scc))
    errs["cq"] = rel_fro(taps["cq"], mm("cq", taps["c"], d, d))
    tx = text_bf.float().cpu().numpy()[trows]
    errs["ckv"] = rel_fro(taps["ckv"], mm("ckv", tx, 2 * d, d))
    errs["co"] = rel_fro(taps["h_co"] - taps["h_o"], gc * mm("co", taps["cq"], d, d))
    errs["a2"] = rel_fro(taps["a2"], norm_mod(taps["h_co"], sh2, sc2))
    errs["fc1_swiglu"] = rel_fro(taps["g"], oracle.swiglu(mm("fc1", taps["a2"], 2 * F, d)))
    errs["fc2"] = rel_fro(taps["h_fc2"] - taps["h_co"], g2 * mm("fc2", taps["g"], d, F))
    bad = {k: v for k, v in errs.items() if not v <= GEMM_TOL}
    assert not bad, (bad, errs)

    # the whole block composed in fp32 from the starting rows
    a = norm_mod(hs, sh1, sc1)
    qkv = mm("qkv", a, 3 * d, d)
    hr = oracle.gate_residual(hs, np.tile(g1, (n, 1)), mm("o", qkv[:, 2 * d:], d, d))
    c = norm_mod(hr, shc, scc)
    hr = oracle.gate_residual(hr, np.tile(gc, (n, 1)), mm("co", mm("cq", c, d, d), d, d))
    a2 = norm_mod(hr, sh2, sc2)
    hr = oracle.gate_residual(hr, np.tile(g2, (n, 1)), mm("fc2", oracle.swiglu(mm("fc1", a2, 2 * F, d)), d, F))
    got = h.cpu().numpy()[rows]
    assert np.array_equal(got, taps["h_fc2"])
    assert rel_fro(got - hs, hr - hs) <= CHAIN_TOL
    assert rel_fro(taps["ckv"], mm("ckv", text.cpu().numpy()[trows], 2 * d, d)) <= CHAIN_TOL


def test_config3_swiglu_ffn_chain(fh3, oracle, default_gemm_path):
    import torch
    d, F, M = 5120, 13824, 4096
    w1 = fh3.make_weights(2 * F, d, seed=0, stream_id=31)      # [W_up; W_gate], value-first
    w2 = fh3.make_weights(d, F, seed=0, stream_id=32)          # W_down
    x = torch.randn((M, d), device="cuda", generator=torch.Generator(device="cuda").manual_seed(43))
    xb = fh3.to_bf16(x)
    gm = fh3.gemm(w1, xb, fh3.EPI_SWIGLU)                      # bf16 [M][F]
    y = fh3.gemm(w2, gm, fh3.EPI_F32)                          # fp32 [M][d]
    torch.cuda.synchronize()
    assert fh3.device_status() == 0
    rows = _sample(M, SAMPLE, 6)
    r1, r2 = w1.data.cpu().numpy(), w2.data.cpu().numpy()
    xs = x.cpu().numpy()[rows]
    xbs = xb.float().cpu().numpy()[rows]
    gs = gm.float().cpu().numpy()[rows]
    ys = y.cpu().numpy()[rows]
    assert np.isfinite(y.cpu().numpy()).all()
    assert rel_fro(gs, oracle.swiglu(oracle.matmul(Q4K, r1, d, 2 * F, xbs))) <= GEMM_TOL
    assert rel_fro(ys, oracle.matmul(Q4K, r2, F, d, gs)) <= GEMM_TOL
    chain = oracle.matmul(Q4K, r2, F, d, oracle.swiglu(oracle.matmul(Q4K, r1, d, 2 * F, xs)))
    assert rel_fro(ys, chain) <= CHAIN_TOL
