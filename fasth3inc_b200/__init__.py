"""fasth3inc_b200 -- B200-native Q4_K dequantise-and-multiply for fh3.

Host-side mirror of the reference's matmul interface (include/fh3/fh3.h:82-109):

    row_bytes(type, n)                     fh3_row_bytes   (src/core/fh3_quant.c:14-34)
    dequant(type, src, n, rows)            fh3_dequant     (src/core/fh3_quant.c:284-318)
    matmul(w, x, bias)                     fh3_matmul      (src/core/fh3_ops.c:317-404)
    matmul_host(w, x, bias)                fh3_matmul on host buffers through the C drop-in

Every call goes through libfh3cuda.so (the C ABI in include/fh3cuda.h) on
device memory owned by torch tensors; torch is only the allocator and stream
provider here.  There is no CPU path: without the CUDA library or a GPU these
functions raise.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import (BF16, EPI_BF16, EPI_F32, EPI_RESID, EPI_SWIGLU, F16, F32, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_0,
                   Fh3CudaError, Fh3CudaW,
                   check, load)

__all__ = [
    "Q4_K", "F32", "F16", "BF16", "Q8_0", "Q2_K", "Q3_K", "Q5_K", "Q6_K", "Weight", "EPI_F32", "EPI_BF16", "EPI_SWIGLU", "EPI_RESID", "Fh3CudaError", "Q4KWeight",
    "init", "row_bytes", "dequant", "matmul", "gemv", "gemm", "matmul_host", "rmsnorm_modulate",
    "to_bf16", "swiglu", "qk_norm_rope", "attention", "vsa_attention", "vsa_tiles", "vsa_num_tiles",
    "make_weights", "device_status",
]

_inited: set[int] = set()


def _torch():
    import torch
    return torch


def init(device: int = 0) -> None:
    """Set up libfh3cuda on `device` (fh3cuda_init)."""
    torch = _torch()
    torch.cuda.set_device(device)
    L = load()
    check(L.fh3cuda_init(device))
    _inited.add(device)


def _ensure(t) -> None:
    dev = t.device.index if t.device.index is not None else _torch().cuda.current_device()
    if dev not in _inited:
        init(dev)


def _stream(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def sm_count() -> int:
    """SMs of the current device (0 before init)."""
    return int(load().fh3cuda_sm_count())


def row_bytes(type_: int, n: int) -> int:
    """Bytes of one row of `n` weights (fh3_row_bytes)."""
    return int(load().fh3cuda_row_bytes(type_, n))


@dataclass
class Q4KWeight:
    """A weight matrix resident in HBM: `out` rows of `in_` weights of format `type`
    (Fh3W; Q4_K unless given)."""
    data: object  # torch.uint8 tensor on the device, out * row_bytes(type, in_) bytes
    in_: int
    out: int
    type: int = Q4_K

    @property
    def desc(self) -> Fh3CudaW:
        return Fh3CudaW(self.type, self.in_, self.out, self.data.data_ptr())

    @property
    def nbytes(self) -> int:
        return self.out * row_bytes(self.type, self.in_)

    @classmethod
    def from_bytes(cls, raw: np.ndarray, in_: int, out: int, device: int | str = "cuda",
                   type_: int = Q4_K) -> "Q4KWeight":
        torch = _torch()
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        if raw.size != out * row_bytes(type_, in_):
            raise ValueError("byte count does not match out * row_bytes(type, in)")
        return cls(torch.from_numpy(raw).to(device), in_, out, type_)


Weight = Q4KWeight  # any format fh3_dequant expands


def dequant(type_: int, src, n: int, rows: int = 1, out=None, stream=None):
    """Dequantise `rows` rows of `n` weights to fp32 (fh3_dequant, bit-exact)."""
    torch = _torch()
    _ensure(src)
    if out is None:
        out = torch.zeros((rows, n), dtype=torch.float32, device=src.device)
    check(load().fh3cuda_dequant_dev(type_, _ptr(src), _ptr(out), rows, n, _stream(stream)))
    return out


def matmul(w: Q4KWeight, x, bias=None, out=None, stream=None):
    """y = x . W^T (+ bias) on device tensors (fh3_matmul semantics)."""
    torch = _torch()
    _ensure(x)
    x = x.contiguous()
    n_tok = x.shape[0]
    if out is None:
        out = torch.empty((n_tok, w.out), dtype=torch.float32, device=x.device)
    d = w.desc
    check(load().fh3cuda_matmul_dev(ctypes.byref(d), _ptr(x), _ptr(out), n_tok, _ptr(bias), _stream(stream)))
    return out


def gemv(w: Q4KWeight, x, bias=None, out=None, stream=None):
    """Q4_K GEMV for 1..16 tokens (fh3cuda_gemv_q4k_dev): tensor-core kernels by default
    (warp-level integer MMAs of the nibbles against digits of x at 1-2 tokens and at 3-4
    when out > in; otherwise tcgen05 MMAs: integer MMAs up to 5 tokens, f16 MMAs of sc*q
    from 6);
    FH3CUDA_GEMV_KERNEL=tc | mma-stream | mma-cta | mma-i8 | fp32 selects one."""
    torch = _torch()
    _ensure(x)
    n_tok = x.shape[0]
    if out is None:
        out = torch.empty((n_tok, w.out), dtype=torch.float32, device=x.device)
    d = w.desc
    check(load().fh3cuda_gemv_q4k_dev(ctypes.byref(d), _ptr(x), _ptr(out), n_tok, _ptr(bias), _stream(stream)))
    return out


def gemm(w: Q4KWeight, x_bf16, epi: int = EPI_F32, bias=None, gate=None, out=None, stream=None):
    """The tcgen05 GEMM on bf16 activations with the chosen epilogue."""
    torch = _torch()
    _ensure(x_bf16)
    n_tok = x_bf16.shape[0]
    n_out = w.out // 2 if epi == EPI_SWIGLU else w.out
    if out is None:
        dt = torch.bfloat16 if epi in (EPI_BF16, EPI_SWIGLU) else torch.float32
        out = torch.empty((n_tok, n_out), dtype=dt, device=x_bf16.device)
    if x_bf16.stride(-1) != 1:
        raise ValueError("x_bf16 rows must be contiguous")
    d = w.desc
    check(load().fh3cuda_gemm_q4k_dev(ctypes.byref(d), _ptr(x_bf16), x_bf16.stride(0), _ptr(out),
                                      out.stride(0), n_tok, _ptr(bias), _ptr(gate), epi, _stream(stream)))
    return out


def q4k_to_bf16(w: Q4KWeight, out=None, stream=None):
    """W's Q4_K rows as bf16 [out][in] (fh3's fp32 weight rounded once): the first half of
    the two-pass GEMM."""
    torch = _torch()
    _ensure(w.data)
    if out is None:
        out = torch.empty((w.out, w.in_), dtype=torch.bfloat16, device=w.data.device)
    d = w.desc
    check(load().fh3cuda_q4k_to_bf16_dev(ctypes.byref(d), _ptr(out), _stream(stream)))
    return out


def gemm_bf16w(w_bf16, x_bf16, epi: int = EPI_F32, bias=None, gate=None, out=None, stream=None,
               weights_ready: bool = False):
    """The tcgen05 GEMM on a bf16 [out][in] weight matrix (fh3cuda_gemm_bf16w_dev): the
    second half of the two-pass GEMM, same epilogues as gemm()."""
    torch = _torch()
    _ensure(x_bf16)
    n_tok = x_bf16.shape[0]
    N, K = w_bf16.shape
    n_out = N // 2 if epi == EPI_SWIGLU else N
    if out is None:
        dt = torch.bfloat16 if epi in (EPI_BF16, EPI_SWIGLU) else torch.float32
        out = torch.empty((n_tok, n_out), dtype=dt, device=x_bf16.device)
    if x_bf16.stride(-1) != 1 or not w_bf16.is_contiguous():
        raise ValueError("x_bf16 rows and the weight matrix must be contiguous")
    check(load().fh3cuda_gemm_bf16w_dev(_ptr(w_bf16), N, K, _ptr(x_bf16), x_bf16.stride(0), _ptr(out),
                                        out.stride(0), n_tok, _ptr(bias), _ptr(gate), epi,
                                        _lib.GEMM_WEIGHTS_READY if weights_ready else 0, _stream(stream)))
    return out


def to_bf16(x, out=None, stream=None):
    torch = _torch()
    _ensure(x)
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    check(load().fh3cuda_f32_to_bf16_dev(_ptr(x), _ptr(out), x.numel(), _stream(stream)))
    return out


def rmsnorm_modulate(x, shift, scale, norm_w=None, eps: float = 1e-6, out=None, stream=None):
    """bf16(modulate(rmsnorm(x))) per row (fh3_rmsnorm + fh3_modulate, fused)."""
    torch = _torch()
    _ensure(x)
    n, dim = x.shape
    if out is None:
        out = torch.empty((n, dim), dtype=torch.bfloat16, device=x.device)
    check(load().fh3cuda_rmsnorm_modulate_dev(_ptr(x), _ptr(norm_w), _ptr(shift), _ptr(scale), _ptr(out),
                                              n, dim, eps, _stream(stream)))
    return out


def qk_norm_rope(src, norm_w, cos=None, sin=None, heads: int = 1, head_dim: int = 128, rot_dim: int = 0,
                 eps: float = 1e-6, out=None, out_bf16: bool = False, stream=None):
    """fh3_rmsnorm per head then fh3_rope3 (fh3_dit.c:397-401) on a [n][>= heads*head_dim]
    fp32 or bf16 view (e.g. the q or k third of a QKV output); returns [n][heads*head_dim]."""
    torch = _torch()
    _ensure(src)
    n = src.shape[0]
    if src.stride(-1) != 1:
        raise ValueError("src rows must be contiguous")
    if out is None:
        dt = torch.bfloat16 if out_bf16 else torch.float32
        out = torch.empty((n, heads * head_dim), dtype=dt, device=src.device)
    check(load().fh3cuda_qk_norm_rope_dev(
        _ptr(src), int(src.dtype == torch.bfloat16), src.stride(0), _ptr(out), int(out.dtype == torch.bfloat16),
        out.stride(0), _ptr(norm_w), _ptr(cos), _ptr(sin), n, heads, head_dim, rot_dim, eps, _stream(stream)))
    return out


def attention(q, k, v, heads: int, head_dim: int = 128, out=None, out_bf16: bool = False, stream=None):
    """fh3_attention on [n][>= heads*head_dim] views (e.g. the thirds of a QKV output); returns
    o [n][heads*head_dim].  bf16 q/k/v run on tensor cores (head_dim 128; o fp32, or bf16 with
    out_bf16); fp32 q/k/v run in fp32 (head_dim a multiple of 32 up to 256; o fp32)."""
    torch = _torch()
    dt = q.dtype
    for t in (q, k, v):
        _ensure(t)
        if t.dtype != dt or dt not in (torch.bfloat16, torch.float32) or t.stride(-1) != 1:
            raise ValueError("q, k, v must share one dtype (bf16 or fp32) with contiguous rows")
    n = q.shape[0]
    f32 = dt == torch.float32
    if out is None:
        out = torch.empty((n, heads * head_dim), dtype=torch.bfloat16 if (out_bf16 and not f32) else torch.float32,
                          device=q.device)
    if f32:
        check(load().fh3cuda_attention_f32_dev(_ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v), v.stride(0),
                                               _ptr(out), out.stride(0), n, heads, head_dim, _stream(stream)))
    else:
        check(load().fh3cuda_attention_dev(_ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v), v.stride(0),
                                           _ptr(out), int(out.dtype == torch.bfloat16), out.stride(0), n, heads,
                                           head_dim, _stream(stream)))
    return out


def vsa_num_tiles(seq, tile: int = 64) -> tuple[int, int, int]:
    """(num_tiles, num_prefix_tiles, num_video_tiles) of seq = (n, T, A, V, grid_t, grid_h, grid_w)."""
    from ._lib import Fh3CudaSeq
    a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(load().fh3cuda_vsa_num_tiles(ctypes.byref(Fh3CudaSeq(*seq)), tile, ctypes.byref(a), ctypes.byref(b),
                                       ctypes.byref(c)))
    return a.value, b.value, c.value


def vsa_attention(q, k, v, gate, seq, heads: int, head_dim: int, tile: int = 64, sparsity: float = 0.8, out=None,
                  out_bf16: bool = False, stream=None):
    """fh3_vsa_attention (src/core/fh3_vsa.c:186-507) on [n][>= heads*head_dim] device views.

    q, k, v (and gate, or None) all fp32 or all bf16; seq = (n, T, A, V, grid_t, grid_h, grid_w)
    as fh3's Fh3Seq; returns o [n][heads*head_dim] (fp32, or bf16 with out_bf16 for bf16 operands).
    The tile mask is the reference's exactly; bf16 operands run the fine pass on tensor cores,
    fp32 operands in fp32."""
    from ._lib import Fh3CudaSeq
    torch = _torch()
    dt = q.dtype
    for t in (q, k, v) + ((gate,) if gate is not None else ()):
        _ensure(t)
        if t.dtype != dt or dt not in (torch.float32, torch.bfloat16) or t.stride(-1) != 1:
            raise ValueError("q, k, v, gate must share one dtype (fp32 or bf16) with contiguous rows")
    n = q.shape[0]
    if out is None:
        out = torch.empty((n, heads * head_dim),
                          dtype=torch.bfloat16 if (out_bf16 and dt == torch.bfloat16) else torch.float32,
                          device=q.device)
    check(load().fh3cuda_vsa_attention_dev(
        tile, sparsity, ctypes.byref(Fh3CudaSeq(*seq)), _ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v),
        v.stride(0), int(dt == torch.bfloat16), _ptr(gate) if gate is not None else None,
        gate.stride(0) if gate is not None else 0, _ptr(out), int(out.dtype == torch.bfloat16), out.stride(0),
        heads, head_dim, _stream(stream)))
    return out


def vsa_tiles(q, k, seq, heads: int, head_dim: int, tile: int = 64, sparsity: float = 0.8, stream=None):
    """The tile stage of vsa_attention: (scores [heads][T][T] fp32, mask [heads][T][T] uint8) on the device."""
    from ._lib import Fh3CudaSeq
    torch = _torch()
    for t in (q, k):
        _ensure(t)
    nt = vsa_num_tiles(seq, tile)[0]
    scores = torch.empty((heads, nt, nt), dtype=torch.float32, device=q.device)
    mask = torch.empty((heads, nt, nt), dtype=torch.uint8, device=q.device)
    check(load().fh3cuda_vsa_tiles_dev(tile, sparsity, ctypes.byref(Fh3CudaSeq(*seq)), _ptr(q), q.stride(0), _ptr(k),
                                       k.stride(0), int(q.dtype == torch.bfloat16), heads, head_dim, _ptr(scores),
                                       _ptr(mask), _stream(stream)))
    return scores, mask


def swiglu(h, out=None, stream=None):
    """fh3_swiglu on a [n, 2F] fp32 device tensor (value-first halves)."""
    torch = _torch()
    _ensure(h)
    n, two_f = h.shape
    if out is None:
        out = torch.empty((n, two_f // 2), dtype=torch.float32, device=h.device)
    check(load().fh3cuda_swiglu_dev(_ptr(h), _ptr(out), n, two_f // 2, _stream(stream)))
    return out


def make_weights(rows: int, n: int, seed: int, stream_id: int, scale: float = 0.02, device="cuda",
                 stream=None) -> Q4KWeight:
    """Seeded synthetic Q4_K weights generated in HBM (benchmark inputs)."""
    torch = _torch()
    data = torch.empty(rows * row_bytes(Q4_K, n), dtype=torch.uint8, device=device)
    _ensure(data)
    check(load().fh3cuda_make_q4k_weights_dev(seed, stream_id, scale, rows, n, _ptr(data), _stream(stream)))
    return Q4KWeight(data, n, rows)


def device_status(stream=None) -> int:
    """Synchronise and read the device status word (FH3_OK or FH3CUDA_E_TIMEOUT)."""
    return int(load().fh3cuda_device_status(_stream(stream)))


def matmul_host(w_raw: np.ndarray, in_: int, out: int, x: np.ndarray, bias: np.ndarray | None = None,
                y: np.ndarray | None = None, type_: int = Q4_K) -> np.ndarray:
    """fh3_matmul on HOST buffers through the C drop-in (fh3cuda_matmul).

    Raises Fh3CudaError with the drop-in's recorded status on failure.
    """
    L = load()
    if not _inited:
        init(_torch().cuda.current_device())
    w_raw = np.ascontiguousarray(w_raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n_tok = x.shape[0] if x.ndim == 2 else 1
    if y is None:
        y = np.empty((n_tok, out), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    d = Fh3CudaW(type_, in_, out, w_raw.ctypes.data)
    L.fh3cuda_matmul(ctypes.byref(d), x.ctypes.data, y.ctypes.data, n_tok,
                     None if b is None else b.ctypes.data)
    rc = L.fh3cuda_take_status()
    if rc != 0:
        raise Fh3CudaError(rc, _lib.last_error())
    return y
