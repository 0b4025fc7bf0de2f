"""Split-K of the fused tcgen05 GEMM for small tile counts (BASELINE config 1's shape: 256 rows,
5120 x 5120 Q4_K weights, 20 tiles of 256 x 256 for 74 CTA pairs; and up to 128 rows, which would
otherwise run one CTA per 256 output columns on the one-SM kernel): the super-blocks of each tile
are cut into ranges, each range's fp32 accumulator is stored, and a reduction adds the ranges in
order and applies the epilogue.  Same values as whole tiles up to fp32 rounding, bit-identical from
call to call, for the fp32, bf16 and gated-residual epilogues; <= 5e-3 against fh3_matmul."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(256, 5120, 5120), (300, 768, 2048), (129, 256, 1024), (200, 100, 256),
                                   (128, 5120, 5120), (40, 300, 1024), (17, 33, 2048)])
def test_split_k_matches_whole_tiles(fh3, oracle, monkeypatch, M, N, K):
    import torch
    monkeypatch.delenv("FH3CUDA_GEMM_KERNEL", raising=False)
    raw = oracle.make_weights(seed=M, stream=17, rows=N, n=K)
    w = fh3.Q4KWeight.from_bytes(raw, K, N)
    x32 = torch.randn((M, K), device="cuda", generator=torch.Generator(device="cuda").manual_seed(M))
    x = fh3.to_bf16(x32)
    bias = torch.randn(N, device="cuda")
    gate = torch.randn(N, device="cuda")
    h0 = torch.randn((M, N), device="cuda")
    outs = {}
    for sk in ("1", "0"):
        monkeypatch.setenv("FH3CUDA_GEMM_SPLITK", sk)
        r = [fh3.gemm(w, x, fh3.EPI_F32, bias=bias), fh3.gemm(w, x, fh3.EPI_BF16, bias=bias)]
        h = h0.clone()
        fh3.gemm(w, x, fh3.EPI_RESID, bias=bias, gate=gate, out=h)
        r.append(h)
        assert torch.equal(fh3.gemm(w, x, fh3.EPI_F32, bias=bias), r[0])      # deterministic
        outs[sk] = r
    # only the fp32 summation order differs (bf16 outputs may then round one ulp apart)
    for a, b, tol in zip(outs["1"], outs["0"], (1e-5, 5e-4, 1e-5)):
        a, b = a.double(), b.double()
        assert ((a - b).norm() / b.norm()).item() <= tol
    ref = oracle.matmul(12, raw, K, N, x.float().cpu().numpy(), bias.cpu().numpy())
    assert rel_fro(outs["1"][0].cpu().numpy(), ref) <= 5e-3
    # the drop-in entry point on fp32 x (config 1 goes through it)
    monkeypatch.setenv("FH3CUDA_GEMM_SPLITK", "1")
    y = fh3.matmul(w, x32, bias)
    assert rel_fro(y.cpu().numpy(), oracle.matmul(12, raw, K, N, x32.cpu().numpy(), bias.cpu().numpy())) <= 5e-3
    assert fh3.device_status() == 0


@pytest.mark.parametrize("M,N", [(256, 1024), (96, 1024), (600, 4096), (2100, 1024)])
def test_dependent_chain_queued_equals_synchronised(fh3, oracle, monkeypatch, M, N):
    """GEMMs that consume the previous GEMM's output, queued back to back (each launched as a
    programmatic dependent of the previous kernel, its weights loaded before the wait, the
    split-K partials reused call after call) give the same bits as the same chain with a
    synchronisation after every call.  Shapes: split-K (256 and 96 rows), whole tiles on the fused
    kernel (600 x 4096), the two-pass path (2100 rows)."""
    import torch
    monkeypatch.delenv("FH3CUDA_GEMM_KERNEL", raising=False)
    K = N
    ws = [fh3.Q4KWeight.from_bytes(oracle.make_weights(seed=200 + i, stream=19, rows=N, n=K), K, N) for i in range(4)]
    g = torch.Generator(device="cuda").manual_seed(M)
    x = fh3.to_bf16(torch.randn((M, K), device="cuda", generator=g))
    gate = torch.randn(N, device="cuda", generator=g)
    h0 = torch.randn((M, N), device="cuda", generator=g)

    def chain(sync):
        h = h0.clone()
        a = fh3.gemm(ws[0], x, fh3.EPI_BF16)
        if sync:
            torch.cuda.synchronize()
        b = fh3.gemm(ws[1], a, fh3.EPI_BF16)            # reads the previous GEMM's output
        if sync:
            torch.cuda.synchronize()
        fh3.gemm(ws[2], b, fh3.EPI_RESID, gate=gate, out=h)  # h += gate * (b W^T), in place
        if sync:
            torch.cuda.synchronize()
        fh3.gemm(ws[3], fh3.to_bf16(h), fh3.EPI_RESID, gate=gate, out=h)
        torch.cuda.synchronize()
        return a, b, h

    ref = chain(True)
    for _ in range(3):
        got = chain(False)
        for r, t in zip(ref, got):
            assert torch.equal(r, t)
    assert fh3.device_status() == 0
