"""The synthetic DiT block (the bench workload) against the same dataflow composed from
the oracle's restatements of fh3_matmul, fh3_rmsnorm, fh3_modulate, fh3_swiglu and
fh3_gate_residual (src/core/fh3_ops.c:317-585), at reduced width."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu
Q4K = 12


def _oracle_block(o, raw, vecs, h, text, d, F):
    n = h.shape[0]
    ones = np.ones(d, np.float32)

    def norm_mod(x, shift, scale):
        return o.modulate(o.rmsnorm(x, ones, 1e-6), np.tile(shift, (n, 1)), np.tile(scale, (n, 1)))

    sh1, sc1, g1, shc, scc, gc, sh2, sc2, g2 = vecs
    a = norm_mod(h, sh1, sc1)
    qkv = o.matmul(Q4K, raw["qkv"], d, 3 * d, a)
    h = o.gate_residual(h, np.tile(g1, (n, 1)), o.matmul(Q4K, raw["o"], d, d, qkv[:, 2 * d:]))
    c = norm_mod(h, shc, scc)
    cq = o.matmul(Q4K, raw["cq"], d, d, c)
    ckv = o.matmul(Q4K, raw["ckv"], d, 2 * d, text)
    h = o.gate_residual(h, np.tile(gc, (n, 1)), o.matmul(Q4K, raw["co"], d, d, cq))
    a2 = norm_mod(h, sh2, sc2)
    g = o.swiglu(o.matmul(Q4K, raw["fc1"], d, 2 * F, a2))
    h = o.gate_residual(h, np.tile(g2, (n, 1)), o.matmul(Q4K, raw["fc2"], F, d, g))
    return h, ckv


def test_two_blocks_match_oracle_composition(fh3, oracle):
    import torch

    from fasth3inc_b200.trunk import Runner, Trunk, Workspace
    d, F, M, T = 512, 1024, 300, 40
    trunk = Trunk(d=d, F=F, n_blocks=2, seed=7).build()
    ws = Workspace(M, T, d=d, F=F)
    g = torch.Generator(device="cuda").manual_seed(3)
    h0 = torch.randn((M, d), device="cuda", generator=g)
    text = torch.randn((T, d), device="cuda", generator=g)
    text_bf = fh3.to_bf16(text)
    h = h0.clone()
    Runner(trunk, ws).step(h, text_bf)
    torch.cuda.synchronize()
    assert fh3.device_status() == 0

    href = h0.cpu().numpy()
    # the GPU feeds bf16 text rows to the K/V projection; give the oracle the same values
    tx = text_bf.float().cpu().numpy()
    for blk in trunk.blocks:
        raw = {k: w.data.cpu().numpy() for k, w in blk.w.items()}
        vecs = [v.cpu().numpy() for v in (blk.shift1, blk.scale1, blk.gate1, blk.shift_c, blk.scale_c,
                                          blk.gate_c, blk.shift2, blk.scale2, blk.gate2)]
        href, ckv = _oracle_block(oracle, raw, vecs, href, tx, d, F)
    got = h.cpu().numpy()
    h0n = h0.cpu().numpy()
    # chained bf16 GEMMs: the residual increment within 1e-2 of the fp32 composition
    assert rel_fro(got - h0n, href - h0n) <= 1e-2
    # last block's text K/V projection (bf16 output)
    assert rel_fro(ws.ckv.float().cpu().numpy(), ckv) <= 5e-3


def test_rows_for_rank_partitions_rows():
    from fasth3inc_b200.trunk import rows_for_rank
    for total in (33784, 7, 1):
        for world in (1, 2, 4, 8):
            spans = [rows_for_rank(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("M", [300, 2500])
def test_queued_step_equals_stage_by_stage(fh3, M):
    """The step queued as the bench runs it (norms and GEMMs chained by programmatic dependent
    launch, every expansion on the side stream one projection ahead) gives the same bits as
    the same launches with a synchronisation after every stage.  2500 rows take the two-pass
    path with its overlapped expansions; 300 rows the fused kernels."""
    import torch

    from fasth3inc_b200.trunk import Runner, Trunk, Workspace
    d, F, T = 512, 1024, 40
    trunk = Trunk(d=d, F=F, n_blocks=2, seed=9).build()
    ws = Workspace(M, T, d=d, F=F)
    g = torch.Generator(device="cuda").manual_seed(5)
    h0 = torch.randn((M, d), device="cuda", generator=g)
    text_bf = fh3.to_bf16(torch.randn((T, d), device="cuda", generator=g))
    runner = Runner(trunk, ws)

    h_sync = h0.clone()
    for blk in trunk.blocks:
        runner.block(blk, h_sync, text_bf, tap=lambda stage, t: torch.cuda.synchronize())
    torch.cuda.synchronize()
    for _ in range(2):
        h = h0.clone()
        runner.step(h, text_bf)
        torch.cuda.synchronize()
        assert torch.equal(h, h_sync)
    assert fh3.device_status() == 0
