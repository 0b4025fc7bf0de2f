"""Dense attention (fh3_attention, src/core/fh3_ops.c:587-695) on the GPU.

The kernels take bf16 q/k/v (fp32 softmax and accumulation, P rounded to bf16 for the
second product), so they are compared with fp32 computations on the SAME bf16-rounded inputs:
the oracle (bitwise equal to the reference, tests/test_oracle.py) and torch's fp32
attention.  The kernel for bf16 operands is tcgen05 (score and output tiles in tensor
memory, two query tiles a CTA).  Tolerance: relative Frobenius error <= 1e-2 (the bf16
operand bar of the chained block test); against the reference's own fp32-input case the
input rounding is included, tolerance 2e-2.  fp32 operands run in fp32 at 1e-5."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(torch.bfloat16)


def _torch_ref(qb, kb, vb, heads, hd=128):
    import torch
    n = qb.shape[0]
    q, k, v = (t.float()[:, :heads * hd].reshape(n, heads, hd).transpose(0, 1) for t in (qb, kb, vb))
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v)   # fp32, scale 1/sqrt(hd)
    return o.transpose(0, 1).reshape(n, heads * hd)


def test_reference_case(fh3, oracle, golden_cases):
    n, H, D = (int(v) for v in golden_cases["attn/dims"])
    q, k, v = (golden_cases[f"attn/{x}"] for x in "qkv")
    qb, kb, vb = _bf16(q), _bf16(k), _bf16(v)
    got = fh3.attention(qb, kb, vb, H).cpu().numpy()
    assert rel_fro(got, golden_cases["attn/y"]) <= 2 * TOL
    same_inputs = oracle.attention(qb.float().cpu().numpy(), kb.float().cpu().numpy(), vb.float().cpu().numpy(), H, D)
    assert rel_fro(got, same_inputs) <= TOL


@pytest.mark.parametrize("n", [1, 63, 64, 65, 127, 129, 300])
def test_tails_vs_oracle(fh3, oracle, n):
    H = 3
    rng = np.random.default_rng(n)
    q, k, v = (rng.standard_normal((n, H * 128)).astype(np.float32) for _ in range(3))
    qb, kb, vb = _bf16(q), _bf16(k), _bf16(v)
    got = fh3.attention(qb, kb, vb, H).cpu().numpy()
    ref = oracle.attention(qb.float().cpu().numpy(), kb.float().cpu().numpy(), vb.float().cpu().numpy(), H, 128)
    assert rel_fro(got, ref) <= TOL


@pytest.mark.parametrize("n,H", [(1000, 4), (3001, 2)])
def test_larger_vs_torch_fp32(fh3, n, H):
    import torch
    g = torch.Generator(device="cuda").manual_seed(n)
    qb, kb, vb = (torch.randn((n, H * 128), device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    got = fh3.attention(qb, kb, vb, H)
    ref = _torch_ref(qb, kb, vb, H)
    assert rel_fro(got.cpu().numpy(), ref.cpu().numpy()) <= TOL


def test_qkv_thirds_strided_and_outputs(fh3):
    """q, k, v read as strided thirds of one bf16 [n][3*inner] QKV output; fp32 and bf16 o,
    o written into a wider buffer (ldo > heads*128)."""
    import torch
    n, H = 517, 5
    inner = H * 128
    g = torch.Generator(device="cuda").manual_seed(7)
    qkv = (torch.randn((n, 3 * inner), device="cuda", generator=g) * 2.0).to(torch.bfloat16)
    q, k, v = qkv[:, :inner], qkv[:, inner:2 * inner], qkv[:, 2 * inner:]
    ref = _torch_ref(q, k, v, H)
    o32 = fh3.attention(q, k, v, H)
    assert rel_fro(o32.cpu().numpy(), ref.cpu().numpy()) <= TOL
    wide = torch.full((n, inner + 64), 7.0, dtype=torch.bfloat16, device="cuda")
    fh3.attention(q, k, v, H, out=wide[:, :inner])
    assert rel_fro(wide[:, :inner].float().cpu().numpy(), ref.cpu().numpy()) <= TOL
    assert torch.all(wide[:, inner:] == 7.0)          # nothing written past the rows


def test_saturated_and_constant_rows(fh3, oracle):
    """Very large scores (one key dominates) and identical keys (uniform weights)."""
    n, H = 130, 2
    rng = np.random.default_rng(5)
    q = rng.standard_normal((n, H * 128)).astype(np.float32) * 8.0
    k = rng.standard_normal((n, H * 128)).astype(np.float32) * 8.0
    v = rng.standard_normal((n, H * 128)).astype(np.float32)
    k[:, 128:] = 1.0                                   # head 1: all keys equal
    qb, kb, vb = _bf16(q), _bf16(k), _bf16(v)
    got = fh3.attention(qb, kb, vb, H).cpu().numpy()
    ref = oracle.attention(qb.float().cpu().numpy(), kb.float().cpu().numpy(), vb.float().cpu().numpy(), H, 128)
    assert np.isfinite(got).all()
    assert rel_fro(got, ref) <= TOL


def test_rejects_bad_arguments(fh3):
    import torch
    x = torch.zeros((8, 256), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(fh3.Fh3CudaError):
        fh3.attention(x, x, x, 4, head_dim=64)        # only head_dim 128
    with pytest.raises(fh3.Fh3CudaError):
        fh3.attention(x[:, 1:], x, x, 1)              # misaligned view


# ---- fp32 operands (fh3cuda_attention_f32_dev): the CPU path's accuracy ----
TOL_F32 = 1e-5


def test_f32_reference_case(fh3, golden_cases):
    n, H, D = (int(v) for v in golden_cases["attn/dims"])
    q, k, v = (golden_cases[f"attn/{x}"] for x in "qkv")
    dev = lambda a: __import__("torch").from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    got = fh3.attention(dev(q), dev(k), dev(v), H, D).cpu().numpy()
    assert rel_fro(got, golden_cases["attn/y"]) <= TOL_F32


@pytest.mark.parametrize("n,H,D", [(1, 1, 128), (18, 2, 128), (65, 3, 64), (130, 2, 256), (40, 1, 32)])
def test_f32_vs_oracle(fh3, oracle, n, H, D):
    import torch
    rng = np.random.default_rng(n * 7 + D)
    q, k, v = (rng.standard_normal((n, H * D)).astype(np.float32) for _ in range(3))
    got = fh3.attention(*(torch.from_numpy(a).cuda() for a in (q, k, v)), H, D).cpu().numpy()
    assert rel_fro(got, oracle.attention(q, k, v, H, D)) <= TOL_F32
