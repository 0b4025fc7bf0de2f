"""The two halves of the two-pass GEMM as separate entry points, and the trunk runner that
overlaps them.

fh3cuda_q4k_to_bf16_dev must write exactly fh3's fp32 weights (dequant_q4_k,
src/core/fh3_quant.c:154-196) rounded once to bf16; fh3cuda_gemm_bf16w_dev on that
matrix must give the same bits as fh3cuda_gemm_q4k_dev's two-pass path (same kernel, same
weights); and the runner that expands the next projection on a second stream while the
current GEMM runs must give the same bits as one fh3cuda_gemm_q4k_dev call a projection.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
Q4K = 12


@pytest.mark.parametrize("N,K", [(1, 256), (300, 1280), (4096, 5120), (5120, 13824)])
def test_expansion_is_the_fp32_weight_rounded_once(fh3, N, K):
    import torch
    w = fh3.make_weights(N, K, seed=9, stream_id=N)
    wb = fh3.q4k_to_bf16(w)
    ref = fh3.dequant(Q4K, w.data, K, N).to(torch.bfloat16)   # bit-exact fp32, then round to nearest even
    assert torch.equal(wb.view(torch.int16), ref.view(torch.int16))
    assert fh3.device_status() == 0


def test_bf16_weight_gemm_equals_two_pass(fh3, monkeypatch):
    import torch
    monkeypatch.setenv("FH3CUDA_GEMM_KERNEL", "two-pass")
    N, K, M = 768, 1280, 2500
    w = fh3.make_weights(N, K, seed=10, stream_id=2)
    wb = fh3.q4k_to_bf16(w)
    x = fh3.to_bf16(torch.randn((M, K), device="cuda"))
    bias = torch.randn(N, device="cuda")
    g = torch.randn(N, device="cuda")
    for epi in (fh3.EPI_F32, fh3.EPI_BF16, fh3.EPI_SWIGLU):
        assert torch.equal(fh3.gemm(w, x, epi, bias=bias), fh3.gemm_bf16w(wb, x, epi, bias=bias)), epi
    h1 = torch.ones((M, N), device="cuda")
    h2 = h1.clone()
    fh3.gemm(w, x, fh3.EPI_RESID, gate=g, out=h1)
    fh3.gemm_bf16w(wb, x, fh3.EPI_RESID, gate=g, out=h2)
    assert torch.equal(h1, h2)
    # a strided activation view (the V third of a QKV row), as the O projection reads it
    qkv = fh3.to_bf16(torch.randn((M, 3 * K), device="cuda"))
    v = qkv[:, 2 * K:]
    assert torch.equal(fh3.gemm(w, v, fh3.EPI_F32), fh3.gemm_bf16w(wb, v, fh3.EPI_F32))
    assert fh3.device_status() == 0


def test_bf16_weight_gemm_rejects_bad_arguments(fh3):
    import torch
    wb = torch.zeros((64, 96), dtype=torch.bfloat16, device="cuda")     # in = 96: not a multiple of 64
    x = torch.zeros((32, 96), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(fh3.Fh3CudaError):
        fh3.gemm_bf16w(wb, x)
    wb = torch.zeros((63, 128), dtype=torch.bfloat16, device="cuda")    # odd rows with SwiGLU
    with pytest.raises(fh3.Fh3CudaError):
        fh3.gemm_bf16w(wb, torch.zeros((32, 128), dtype=torch.bfloat16, device="cuda"), fh3.EPI_SWIGLU)


def test_overlapped_runner_equals_one_call_a_projection(fh3, monkeypatch):
    import torch

    from fasth3inc_b200 import _lib
    from fasth3inc_b200.trunk import Runner, Trunk, Workspace
    monkeypatch.delenv("FH3CUDA_GEMM_KERNEL", raising=False)
    d, F, M, T = 512, 1024, 2300, 40
    assert _lib.load().fh3cuda_gemm_launches(M) == 2
    trunk = Trunk(d=d, F=F, n_blocks=3, seed=13).build()
    ws = Workspace(M, T, d=d, F=F)
    g = torch.Generator(device="cuda").manual_seed(5)
    h0 = torch.randn((M, d), device="cuda", generator=g)
    text_bf = fh3.to_bf16(torch.randn((T, d), device="cuda", generator=g))
    outs = []
    for overlap in (True, False, True):
        h = h0.clone()
        r = Runner(trunk, ws, overlap=overlap)
        r.step(h, text_bf)
        r.step(h, text_bf)          # a second step reuses the buffers and events
        torch.cuda.synchronize()
        outs.append(h)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    assert np.isfinite(outs[0].cpu().numpy()).all()
    assert fh3.device_status() == 0
