"""Synthetic DiT trunk built on libfh3cuda: the BASELINE workload for the Q4_K path.

Each block issues the same projections the reference's DiT sends through
fh3_matmul (src/model/fh3_dit.c:385-439: rmsnorm+modulate, qkv, out, fc1 with
value-first [up; gate] halves, swiglu, fc2, gated residuals) plus the cross-
attention projections of the BASELINE configuration (Q/O on the latents, K/V on
512 text rows).  Attention itself is outside this path (dense/VSA attention,
src/core/fh3_ops.c:587-695 and src/core/fh3_vsa.c, are later work): the V third
of the QKV output stands in for the self-attention output and the cross Q
projection for the cross-attention output, so every GEMM runs at its real
shape on real data.

Per block (d = 5120, F = 13824, M latent rows, T text rows):
    a   = bf16(modulate(rmsnorm(h), shift1, scale1))
    qkv = a . Wqkv^T                      [M, 3d]  bf16 epilogue
    h  += gate1 * (v . Wo^T)              [M, d]   residual epilogue (v = qkv[:, 2d:])
    c   = bf16(modulate(rmsnorm(h), shift_c, scale_c))
    cq  = c . Wcq^T                       [M, d]   bf16 epilogue
    ckv = text . Wckv^T                   [T, 2d]  bf16 epilogue
    h  += gate_c * (cq . Wco^T)           [M, d]   residual epilogue
    a2  = bf16(modulate(rmsnorm(h), shift2, scale2))
    g   = swiglu(a2 . Wfc1^T)             [M, F]   SwiGLU epilogue
    h  += gate2 * (g . Wfc2^T)            [M, d]   residual epilogue

Token rows are independent in every projection, so a step shards by rows
across GPUs (rows_for_rank); the text K/V projection is computed on every rank.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

from . import (EPI_BF16, EPI_RESID, EPI_SWIGLU, Q4KWeight, _lib, check, init, make_weights, row_bytes,
               Q4_K)

D_MODEL = 5120
N_HEADS = 40
HEAD_DIM = 128
FFN = 13824
TEXT_ROWS = 512
VIDEO_ROWS = 32760
AUDIO_ROWS = 1024
N_BLOCKS = 50

# (name, out rows, in) of one block's projections
def block_shapes(d: int = D_MODEL, F: int = FFN):
    return [("qkv", 3 * d, d), ("o", d, d), ("cq", d, d), ("ckv", 2 * d, d), ("co", d, d),
            ("fc1", 2 * F, d), ("fc2", d, F)]


def block_flops(M: int, T: int, d: int = D_MODEL, F: int = FFN) -> int:
    """GEMM FLOPs of one block: 2*rows*in*out per projection."""
    f = 0
    for name, out, inn in block_shapes(d, F):
        rows = T if name == "ckv" else M
        f += 2 * rows * inn * out
    return f


def block_weight_bytes(d: int = D_MODEL, F: int = FFN) -> int:
    return sum(out * row_bytes(Q4_K, inn) for _, out, inn in block_shapes(d, F))


def rows_for_rank(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous row shard [start, stop) of `total` rows for `rank` of `world` (balanced)."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class Block:
    w: dict
    shift1: object
    scale1: object
    gate1: object
    shift_c: object
    scale_c: object
    gate_c: object
    shift2: object
    scale2: object
    gate2: object


@dataclass
class Trunk:
    """n_blocks blocks of Q4_K weights resident in HBM (generated on the device)."""
    d: int = D_MODEL
    F: int = FFN
    n_blocks: int = N_BLOCKS
    seed: int = 0
    device: int = 0
    blocks: list = field(default_factory=list)

    def build(self) -> "Trunk":
        import torch
        init(self.device)
        dev = f"cuda:{self.device}"
        g = torch.Generator(device=dev).manual_seed(self.seed + 12345)
        for b in range(self.n_blocks):
            ws = {}
            for i, (name, out, inn) in enumerate(block_shapes(self.d, self.F)):
                ws[name] = make_weights(out, inn, seed=self.seed, stream_id=1000 * b + i, scale=0.02, device=dev)
            vec = [0.1 * torch.randn(self.d, device=dev, generator=g) for _ in range(9)]
            self.blocks.append(Block(ws, *vec))
        torch.cuda.synchronize(self.device)
        return self

    @property
    def weight_bytes(self) -> int:
        return self.n_blocks * block_weight_bytes(self.d, self.F)


class Workspace:
    """Activation buffers for M latent rows and T text rows (reused every step)."""

    def __init__(self, M: int, T: int, d: int = D_MODEL, F: int = FFN, device: int = 0):
        import torch
        dev = f"cuda:{device}"
        bf = torch.bfloat16
        self.M, self.T = M, T
        self.a = torch.empty((M, d), dtype=bf, device=dev)
        self.qkv = torch.empty((M, 3 * d), dtype=bf, device=dev)
        self.cq = torch.empty((M, d), dtype=bf, device=dev)
        self.ckv = torch.empty((T, 2 * d), dtype=bf, device=dev)
        self.g = torch.empty((M, F), dtype=bf, device=dev)


class Runner:
    """Launches one block / one step through the C ABI, optionally timing GEMMs with events."""

    def __init__(self, trunk: Trunk, ws: Workspace, stream=None):
        import torch
        self.t = trunk
        self.ws = ws
        self.L = _lib.load()
        self.stream = stream if stream is not None else torch.cuda.current_stream(trunk.device)
        self.s = self.stream.cuda_stream
        self.gemm_events: list | None = None  # list of (start, end, flops) when recording
        self.launches = 0

    def _gemm(self, w: Q4KWeight, x, ldx: int, rows: int, y, ldy: int, epi: int, gate=None):
        import torch
        d = w.desc
        rec = self.gemm_events is not None
        if rec:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
        check(self.L.fh3cuda_gemm_q4k_dev(ctypes.byref(d), x, ldx, y, ldy, rows, None,
                                          None if gate is None else gate.data_ptr(), epi, self.s))
        if rec:
            e1.record(self.stream)
            self.gemm_events.append((e0, e1, 2 * rows * w.in_ * w.out))
        self.launches += self.L.fh3cuda_gemm_launches(rows)

    def _norm(self, h, shift, scale, out):
        check(self.L.fh3cuda_rmsnorm_modulate_dev(h.data_ptr(), None, shift.data_ptr(), scale.data_ptr(),
                                                  out.data_ptr(), h.shape[0], h.shape[1], 1e-6, self.s))
        self.launches += 1

    def block(self, blk: Block, h, text_bf16) -> None:
        ws, d = self.ws, self.t.d
        M, T = h.shape[0], text_bf16.shape[0]
        W = blk.w
        self._norm(h, blk.shift1, blk.scale1, ws.a)
        self._gemm(W["qkv"], ws.a.data_ptr(), d, M, ws.qkv.data_ptr(), 3 * d, EPI_BF16)
        v = ws.qkv.data_ptr() + 2 * d * 2  # V third of each row (bf16)
        self._gemm(W["o"], v, 3 * d, M, h.data_ptr(), d, EPI_RESID, blk.gate1)
        self._norm(h, blk.shift_c, blk.scale_c, ws.a)
        self._gemm(W["cq"], ws.a.data_ptr(), d, M, ws.cq.data_ptr(), d, EPI_BF16)
        self._gemm(W["ckv"], text_bf16.data_ptr(), d, T, ws.ckv.data_ptr(), 2 * d, EPI_BF16)
        self._gemm(W["co"], ws.cq.data_ptr(), d, M, h.data_ptr(), d, EPI_RESID, blk.gate_c)
        self._norm(h, blk.shift2, blk.scale2, ws.a)
        self._gemm(W["fc1"], ws.a.data_ptr(), d, M, ws.g.data_ptr(), self.t.F, EPI_SWIGLU)
        self._gemm(W["fc2"], ws.g.data_ptr(), self.t.F, M, h.data_ptr(), d, EPI_RESID, blk.gate2)

    def step(self, h, text_bf16) -> None:
        """One denoising step of the trunk on the rows of h (fp32, updated in place)."""
        for blk in self.t.blocks:
            self.block(blk, h, text_bf16)
