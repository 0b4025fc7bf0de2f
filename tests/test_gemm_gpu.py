"""The tcgen05 Q4_K GEMM (bf16 operands, fp32 accumulation) against fh3_matmul.

Tolerance: relative Frobenius error <= 5e-3 for the bf16
tensor-core path.  References: the reference's own outputs (tests/golden), the
oracle (bitwise equal to fh3_matmul), and a plain PyTorch fp64 matmul on the
bit-exact dequantised weights for shapes the CPU oracle would take long on.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import read_matmul_golden, rel_fro

pytestmark = pytest.mark.gpu
Q4K = 12
TOL = 5e-3


@pytest.fixture(autouse=True, params=["2sm", "1sm", "two-pass"])
def gemm_kernel(request, monkeypatch):
    """Run every test on every GEMM path: the fused CTA-pair (cta_group::2) kernel that serves
    128 < M < 2048 by default, the fused one-SM kernel (M <= 128), and the two-pass path of
    M >= 2048 (weights dequantised to bf16 once per call, then the TMA-fed bf16 pair kernel)."""
    monkeypatch.setenv("FH3CUDA_GEMM_KERNEL", request.param)
    return request.param


def _w(fh3, raw, K, N):
    return fh3.Q4KWeight.from_bytes(raw, K, N)


def _torch_ref(fh3, w, x, bias=None):
    """fp64 x . dequant(W)^T (+ bias) with W dequantised bit-exactly on the GPU."""
    import torch
    wf = fh3.dequant(Q4K, w.data, w.in_, w.out).double()
    y = x.double() @ wf.T
    if bias is not None:
        y = y + bias.double()
    return y


def test_reference_cases_through_matmul(fh3, golden_cases):
    import torch
    seen = 0
    for name in sorted({k.split("/")[0] for k in golden_cases if k.startswith("k")}):
        K, N, M = (int(v) for v in golden_cases[f"{name}/dims"])
        if M <= 16:
            continue
        w = _w(fh3, golden_cases[f"{name}/w"], K, N)
        x = torch.from_numpy(golden_cases[f"{name}/x"]).cuda()
        b = golden_cases.get(f"{name}/bias")
        bt = None if b is None else torch.from_numpy(b).cuda()
        y = fh3.matmul(w, x, bt).cpu().numpy()
        assert rel_fro(y, golden_cases[f"{name}/y"]) <= TOL, name
        seen += 1
    assert seen >= 2


def test_reference_fp64_golden(fh3):
    import torch
    t, K, N, M, w, x, bias, y = read_matmul_golden()
    got = fh3.matmul(_w(fh3, w, K, N), torch.from_numpy(x).cuda(), torch.from_numpy(bias).cuda())
    assert rel_fro(got.cpu().numpy(), y) <= TOL


def test_config1_gemm_vs_oracle(fh3, oracle):
    import torch
    K = N = 5120
    M = 256
    raw = oracle.make_weights(seed=0, stream=1, rows=N, n=K)
    x = oracle.rng_normal(0, 2, M * K).reshape(M, K)
    ref = oracle.matmul(Q4K, raw, K, N, x)
    got = fh3.matmul(_w(fh3, raw, K, N), torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_fro(got, ref) <= TOL


@pytest.mark.parametrize("M,N,K", [(17, 1, 256), (129, 255, 512), (300, 264, 256), (128, 256, 1024),
                                   (513, 700, 768)])
def test_tails_vs_torch(fh3, M, N, K):
    import torch
    w = fh3.make_weights(N, K, seed=M * 31 + N, stream_id=4)
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn((M, K), device="cuda", generator=g)
    b = torch.randn((N,), device="cuda", generator=g)
    got = fh3.matmul(w, x, b)
    ref = _torch_ref(fh3, w, x, b)
    assert rel_fro(got.cpu().numpy(), ref.cpu().numpy()) <= TOL


def test_epilogues_bf16_and_residual(fh3):
    import torch
    M, N, K = 300, 520, 1024
    w = fh3.make_weights(N, K, seed=9, stream_id=1)
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn((M, K), device="cuda", generator=g)
    b = torch.randn((N,), device="cuda", generator=g)
    xb = fh3.to_bf16(x)
    y32 = fh3.gemm(w, xb, fh3.EPI_F32, bias=b)
    y16 = fh3.gemm(w, xb, fh3.EPI_BF16, bias=b)
    torch.cuda.synchronize()
    # same accumulator, same bias add: the bf16 epilogue is the rounded fp32 one
    assert torch.equal(y16, y32.to(torch.bfloat16))
    h0 = torch.randn((M, N), device="cuda", generator=g)
    gate = 0.1 * torch.randn((N,), device="cuda", generator=g)
    h = h0.clone()
    fh3.gemm(w, xb, fh3.EPI_RESID, bias=b, gate=gate, out=h)
    ref = _torch_ref(fh3, w, x, b)
    assert rel_fro((h - h0).cpu().numpy(), (gate.double() * ref).cpu().numpy()) <= TOL
    # bitwise determinism across launches
    again = fh3.gemm(w, xb, fh3.EPI_F32, bias=b)
    assert torch.equal(again, y32)


@pytest.mark.parametrize("F", [256, 200])
def test_swiglu_epilogue_vs_oracle(fh3, oracle, F):
    import torch
    M, K = 150, 512
    raw = oracle.make_weights(seed=F, stream=3, rows=2 * F, n=K)  # [up; gate], value-first
    x = oracle.rng_normal(F, 4, M * K).reshape(M, K)
    h = oracle.matmul(Q4K, raw, K, 2 * F, x)
    ref = oracle.swiglu(h)
    w = _w(fh3, raw, K, 2 * F)
    got = fh3.gemm(w, fh3.to_bf16(torch.from_numpy(x).cuda()), fh3.EPI_SWIGLU)
    assert got.shape == (M, F)
    assert rel_fro(got.float().cpu().numpy(), ref) <= TOL


def test_ffn_sized_gemm_vs_torch(fh3):
    """Config-3 fc1 shape (M 4096, K 5120, N 27648): full-size check against torch fp64."""
    import torch
    M, K, N = 4096, 5120, 27648
    w = fh3.make_weights(N, K, seed=3, stream_id=7)
    x = torch.randn((M, K), device="cuda", generator=torch.Generator(device="cuda").manual_seed(3))
    got = fh3.matmul(w, x)
    ref = _torch_ref(fh3, w, x)
    assert rel_fro(got.cpu().numpy(), ref.cpu().numpy()) <= TOL
    assert fh3.device_status() == 0


def test_rejects_bad_arguments(fh3):
    import torch
    w = fh3.make_weights(64, 256, seed=1, stream_id=1)
    xb = torch.zeros((32, 256), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(fh3.Fh3CudaError):
        fh3.gemm(w, xb, 7)
    with pytest.raises(fh3.Fh3CudaError):
        fh3.gemm(w, xb, fh3.EPI_RESID)  # residual without a gate
    bad = fh3.Q4KWeight(w.data, 320, 64)
    with pytest.raises(fh3.Fh3CudaError):
        fh3.gemm(bad, torch.zeros((32, 320), dtype=torch.bfloat16, device="cuda"))


def test_two_pass_equals_fused_bitwise(fh3, monkeypatch):
    """Both paths feed the tensor cores the same bf16 weights (fh3's fp32 weight rounded once) in
    the same shared-memory layout, MMA shape and k order, so their outputs are identical."""
    import torch
    N, K, M = 1000, 1280, 4200
    w = fh3.make_weights(N, K, seed=5, stream_id=2)
    x = fh3.to_bf16(torch.randn((M, K), device="cuda"))
    g = torch.randn(N, device="cuda")
    outs = {}
    for kern in ("2sm", "two-pass"):
        monkeypatch.setenv("FH3CUDA_GEMM_KERNEL", kern)
        y = fh3.gemm(w, x, fh3.EPI_F32)
        yb = fh3.gemm(w, x, fh3.EPI_BF16)
        h = torch.ones((M, N), device="cuda")
        fh3.gemm(w, x, fh3.EPI_RESID, gate=g, out=h)
        w2 = fh3.make_weights(2 * 512, K, seed=6, stream_id=2)
        ys = fh3.gemm(w2, x, fh3.EPI_SWIGLU)
        outs[kern] = (y, yb, h, ys)
    for a, b in zip(outs["2sm"], outs["two-pass"]):
        assert torch.equal(a, b)


def test_non_finite_activations(fh3, oracle):
    """An Inf or NaN in a row of x makes every output of that row non-finite, as in
    fh3_matmul; the other rows are unaffected (also through a split-K reduction)."""
    import torch
    K, N, M = 1280, 300, 40
    raw = oracle.make_weights(seed=14, stream=1, rows=N, n=K)
    x = oracle.rng_normal(14, 2, M * K).reshape(M, K).astype(np.float32)
    x[3, 100] = np.inf
    x[17, 1000] = np.nan
    with np.errstate(invalid="ignore", over="ignore"):
        ref = oracle.matmul(Q4K, raw, K, N, x)
    got = fh3.matmul(_w(fh3, raw, K, N), torch.from_numpy(x).cuda()).cpu().numpy()
    for r in range(M):
        if r in (3, 17):
            assert not np.isfinite(ref[r]).any() and not np.isfinite(got[r]).any(), r
        else:
            assert rel_fro(got[r], ref[r]) <= TOL, r
