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
    """Launches one block / one step through the C ABI, optionally timing launches with events.

    With `overlap` (the default), every projection of 2048 rows or more runs as its two
    halves: the Q4_K -> bf16 expansion of its weights (fh3cuda_q4k_to_bf16_dev) on a side
    stream into one of two bf16 buffers, and the GEMM on that buffer
    (fh3cuda_gemm_bf16w_dev) on the main stream.  The expansion of the next such
    projection is issued before the current GEMM, waiting only for the GEMM that last
    read its buffer, so it runs while the current GEMM runs: the expansion (HBM-bound)
    leaves the critical path, which the GEMM (tensor-bound) holds.  The launches, the
    bf16 weights and the results are the same as fh3cuda_gemm_q4k_dev's two-pass path.
    Without `overlap` every projection is one fh3cuda_gemm_q4k_dev call."""

    def __init__(self, trunk: Trunk, ws: Workspace, stream=None, overlap: bool = True):
        import torch
        self.t = trunk
        self.ws = ws
        self.L = _lib.load()
        self.stream = stream if stream is not None else torch.cuda.current_stream(trunk.device)
        self.s = self.stream.cuda_stream
        self.overlap = overlap
        self.side = torch.cuda.Stream(device=trunk.device) if overlap else None
        self.wbuf = None                        # two bf16 weight buffers (allocated on first use)
        self.ev_exp = [torch.cuda.Event(), torch.cuda.Event()]
        self.ev_use = [torch.cuda.Event(), torch.cuda.Event()]
        # timing records when not None: lists of (start, end, flops or bytes)
        self.gemm_events: list | None = None
        self.expand_events: list | None = None
        self.norm_events: list | None = None
        self.launches = 0

    # -- one launch each --------------------------------------------------------------
    def _timed(self, kind: str, stream, amount: int, tag: str = ""):
        import torch
        rec = getattr(self, kind)
        if rec is None:
            return None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        rec.append((e0, e1, amount, tag))
        return e1

    def _gemm_fused(self, op):
        w, x, ldx, rows, y, ldy, epi, gate = op[1:9]
        d = w.desc
        e1 = self._timed("gemm_events", self.stream, 2 * rows * w.in_ * w.out, f"fused:{rows}")
        check(self.L.fh3cuda_gemm_q4k_dev(ctypes.byref(d), x, ldx, y, ldy, rows, None,
                                          None if gate is None else gate.data_ptr(), epi, self.s))
        if e1 is not None:
            e1.record(self.stream)
        self.launches += self.L.fh3cuda_gemm_launches(rows)

    def _expand(self, w: Q4KWeight, slot: int):
        """Issue w's expansion into buffer `slot` on the side stream."""
        import torch
        if self.wbuf is None:
            big = max(out * inn for _, out, inn in block_shapes(self.t.d, self.t.F))
            self.wbuf = [torch.empty(big, dtype=torch.bfloat16, device=self.stream.device) for _ in range(2)]
        self.side.wait_event(self.ev_use[slot])          # the GEMM that last read this buffer
        e1 = self._timed("expand_events", self.side, w.out * (row_bytes(Q4_K, w.in_) + 2 * w.in_))
        d = w.desc
        check(self.L.fh3cuda_q4k_to_bf16_dev(ctypes.byref(d), self.wbuf[slot].data_ptr(), self.side.cuda_stream))
        if e1 is not None:
            e1.record(self.side)
        self.ev_exp[slot].record(self.side)
        self.launches += 1

    def _gemm_expanded(self, op, slot: int):
        w, x, ldx, rows, y, ldy, epi, gate = op[1:9]
        self.stream.wait_event(self.ev_exp[slot])
        e1 = self._timed("gemm_events", self.stream, 2 * rows * w.in_ * w.out, f"bf16w:{rows}")
        # the weights were expanded on the side stream and waited for: ready before the previous kernel
        check(self.L.fh3cuda_gemm_bf16w_dev(self.wbuf[slot].data_ptr(), w.out, w.in_, x, ldx, y, ldy, rows, None,
                                            None if gate is None else gate.data_ptr(), epi, _lib.GEMM_WEIGHTS_READY,
                                            self.s))
        if e1 is not None:
            e1.record(self.stream)
        self.ev_use[slot].record(self.stream)
        self.launches += 1

    def _norm(self, op):
        h, shift, scale, out = op[1:5]
        e1 = self._timed("norm_events", self.stream, h.numel() * 4 + out.numel() * 2)
        check(self.L.fh3cuda_rmsnorm_modulate_dev(h.data_ptr(), None, shift.data_ptr(), scale.data_ptr(),
                                                  out.data_ptr(), h.shape[0], h.shape[1], 1e-6, self.s))
        if e1 is not None:
            e1.record(self.stream)
        self.launches += 1

    # -- a block as a list of launches --------------------------------------------------
    def _block_ops(self, blk: Block, h, text_bf16) -> list:
        """One block's launches: ("norm", h, shift, scale, out, tap) and
        ("gemm", w, x, ldx, rows, y, ldy, epi, gate, tap), tap = (stage name, tensor)."""
        ws, d, F = self.ws, self.t.d, self.t.F
        M, T = h.shape[0], text_bf16.shape[0]
        W = blk.w
        v = ws.qkv.data_ptr() + 2 * d * 2  # V third of each row (bf16)
        return [
            ("norm", h, blk.shift1, blk.scale1, ws.a, ("a1", ws.a)),
            ("gemm", W["qkv"], ws.a.data_ptr(), d, M, ws.qkv.data_ptr(), 3 * d, EPI_BF16, None, ("qkv", ws.qkv)),
            ("gemm", W["o"], v, 3 * d, M, h.data_ptr(), d, EPI_RESID, blk.gate1, ("h_o", h)),
            ("norm", h, blk.shift_c, blk.scale_c, ws.a, ("c", ws.a)),
            ("gemm", W["cq"], ws.a.data_ptr(), d, M, ws.cq.data_ptr(), d, EPI_BF16, None, ("cq", ws.cq)),
            ("gemm", W["ckv"], text_bf16.data_ptr(), d, T, ws.ckv.data_ptr(), 2 * d, EPI_BF16, None,
             ("ckv", ws.ckv)),
            ("gemm", W["co"], ws.cq.data_ptr(), d, M, h.data_ptr(), d, EPI_RESID, blk.gate_c, ("h_co", h)),
            ("norm", h, blk.shift2, blk.scale2, ws.a, ("a2", ws.a)),
            ("gemm", W["fc1"], ws.a.data_ptr(), d, M, ws.g.data_ptr(), F, EPI_SWIGLU, None, ("g", ws.g)),
            ("gemm", W["fc2"], ws.g.data_ptr(), F, M, h.data_ptr(), d, EPI_RESID, blk.gate2, ("h_fc2", h)),
        ]

    def _two_pass(self, op) -> bool:
        """Expanded-weight GEMM: every projection of the two-pass row range, and with the
        overlap also the 512-row text K/V projection (its expansion is hidden, and the bf16
        kernel runs its 80 tiles without dequantiser warps)."""
        return self.overlap and op[0] == "gemm" and (op[4] >= self.EXPAND_ROWS or
                                                      self.L.fh3cuda_gemm_launches(op[4]) == 2)

    EXPAND_ROWS = 256

    def run(self, ops: list, tap=None) -> None:
        """Issue `ops` in order; two-pass GEMMs get their expansions one projection ahead.
        No expansion starts before the main stream reaches this call.  Besides "norm" and
        "gemm", an op may be ("call", fn): fn(stream) issues other launches on the main stream
        at that point of the sequence (for example converting the next input to bf16)."""
        import torch
        expanded = [i for i, op in enumerate(ops) if self._two_pass(op)]
        nxt = 0
        if expanded:
            start = torch.cuda.Event()
            start.record(self.stream)
            self.side.wait_event(start)
            self._expand(ops[expanded[0]][1], 0)
        for i, op in enumerate(ops):
            if op[0] == "call":          # ("call", fn): fn(stream) issues its own launches, in order
                op[1](self.stream)
                continue
            if op[0] == "norm":
                self._norm(op)
            elif nxt < len(expanded) and expanded[nxt] == i:
                if nxt + 1 < len(expanded):
                    self._expand(ops[expanded[nxt + 1]][1], (nxt + 1) % 2)
                self._gemm_expanded(op, nxt % 2)
                nxt += 1
            else:
                self._gemm_fused(op)
            if tap is not None:
                tap(*op[-1])

    def block(self, blk: Block, h, text_bf16, tap=None) -> None:
        """One block on the rows of h.  `tap(stage, tensor)`, when given, sees every
        intermediate right after the launch that produces it (the parity tests sample
        rows of each; the launches are the same with or without it)."""
        self.run(self._block_ops(blk, h, text_bf16), tap)

    def step(self, h, text_bf16) -> None:
        """One denoising step of the trunk on the rows of h (fp32, updated in place)."""
        ops = []
        for blk in self.t.blocks:
            ops += self._block_ops(blk, h, text_bf16)
        self.run(ops)
