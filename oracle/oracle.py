"""ctypes front end of the CPU parity oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs import this module, as the checker or as the timed CPU baseline.  The
product (fasth3inc_b200, libfh3cuda) never imports it.

Two libraries sit behind it:
  * ``liboracle.so``       -- this project's C restatement (oracle/fh3_oracle.c),
                              built by ``make -C oracle``; always available.
  * ``_ref/libfh3ref.so``  -- the reference's own fh3_quant.c / fh3_ops.c /
                              fh3_vsa.c / fh3_sched.c compiled from its sources by the same
                              Makefile, where the reference tree exists.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libfh3ref.so")


def reference_tree() -> str | None:
    """The reference's source tree, where this machine has it: $FH3_REF_TREE, else the
    reference_path recorded in the project's BASELINE.json; None when neither exists (GPU
    boxes use the objects built beforehand into _ref/)."""
    cand = os.environ.get("FH3_REF_TREE")
    if not cand:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                cand = json.load(f).get("reference_path")
        except (OSError, ValueError):
            cand = None
    return cand if cand and os.path.isfile(os.path.join(cand, "src", "core", "fh3_ops.c")) else None


REF_TREE = reference_tree()

Q4K = 12
F32 = 0
Q4K_BLOCK = 256
Q4K_BYTES = 144

_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_u8p = ctypes.POINTER(ctypes.c_uint8)


def build(quiet: bool = True, relink: bool = False) -> None:
    """Compile liboracle.so, and where the reference tree exists _ref/libfh3ref.so (and with
    `relink` the fh3 callers relinked against libfh3cuda.so, which must be built first)."""
    cmd = ["make", "-C", HERE] + ([f"REF={REF_TREE}"] if REF_TREE else [])
    out = subprocess.run(cmd + (["all", "relink"] if relink else []), capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(ct) if a is not None else None


class _Fh3W(ctypes.Structure):
    """Mirror of the reference's Fh3W (include/fh3/fh3.h:82-87)."""
    _fields_ = [("type", ctypes.c_int), ("in_", ctypes.c_int64),
                ("out", ctypes.c_int64), ("data", _c_u8p)]


class _Fh3Seq(ctypes.Structure):
    """Mirror of the reference's struct Fh3Seq (src/model/fh3_seq.h:31-45)."""
    _fields_ = [("seq_len", ctypes.c_int), ("num_text", ctypes.c_int), ("num_audio", ctypes.c_int),
                ("num_video", ctypes.c_int), ("grid_t", ctypes.c_int), ("grid_h", ctypes.c_int),
                ("grid_w", ctypes.c_int), ("tags", ctypes.c_void_p), ("pair_index", ctypes.c_void_p),
                ("pos", ctypes.c_void_p), ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p)]


class _Fh3SeqSpec(ctypes.Structure):
    """Mirror of the reference's Fh3SeqSpec (src/model/fh3_seq.h:13-29)."""
    _fields_ = [(n, ctypes.c_int) for n in ("num_text", "num_audio", "num_video", "latent_frames", "latent_height",
                                            "latent_width", "patch_t", "patch_h", "patch_w", "audio_latents",
                                            "audio_channels")] + [
        ("custom_pos", ctypes.c_void_p), ("grid_t", ctypes.c_int), ("grid_h", ctypes.c_int), ("grid_w", ctypes.c_int)]


class _Fh3VsaCfg(ctypes.Structure):
    """Mirror of the reference's Fh3VsaCfg (include/fh3/fh3.h:41-44)."""
    _fields_ = [("tile", ctypes.c_int), ("sparsity", ctypes.c_float)]


class Oracle:
    """This project's C restatement of the reference path."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        lib.oracle_row_bytes.restype = ctypes.c_size_t
        lib.oracle_row_bytes.argtypes = [ctypes.c_int, ctypes.c_int64]
        lib.oracle_dequant_q4k.argtypes = [_c_u8p, _c_f32p, ctypes.c_int64]
        lib.oracle_dequant.restype = ctypes.c_int
        lib.oracle_dequant.argtypes = [ctypes.c_int, _c_u8p, _c_f32p, ctypes.c_int64]
        lib.oracle_matmul.restype = ctypes.c_int
        lib.oracle_matmul.argtypes = [ctypes.c_int, _c_u8p, ctypes.c_int64, ctypes.c_int64,
                                      _c_f32p, _c_f32p, ctypes.c_int, _c_f32p]
        lib.oracle_swiglu.argtypes = [_c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int]
        lib.oracle_rmsnorm.argtypes = [_c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        lib.oracle_modulate.argtypes = [_c_f32p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int]
        lib.oracle_rope3.argtypes = [_c_f32p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int]
        lib.oracle_attention.argtypes = [_c_f32p, _c_f32p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int]
        lib.oracle_gate_residual.argtypes = [_c_f32p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int]
        lib.oracle_rng_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, _c_f32p, ctypes.c_size_t]
        lib.oracle_quantize_q4k.restype = ctypes.c_int
        lib.oracle_quantize_q4k.argtypes = [_c_f32p, _c_u8p, ctypes.c_int64, ctypes.c_int64]
        lib.oracle_make_q4k_weights.restype = ctypes.c_int
        lib.oracle_make_q4k_weights.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float,
                                                ctypes.c_int64, ctypes.c_int64, _c_u8p]
        lib.oracle_num_threads.restype = ctypes.c_int
        lib.oracle_vsa_tiles.restype = ctypes.c_int
        lib.oracle_vsa_tiles.argtypes = [ctypes.c_int] * 8 + [ctypes.POINTER(ctypes.c_int)]
        lib.oracle_vsa.restype = ctypes.c_int
        lib.oracle_vsa.argtypes = ([ctypes.c_int, ctypes.c_float] + [_c_f32p] * 5 + [ctypes.c_int] * 9 +
                                   [_c_f32p, _c_u8p])
        self.lib = lib

    def row_bytes(self, type_: int, n: int) -> int:
        return int(self.lib.oracle_row_bytes(type_, n))

    def dequant_q4k(self, raw: np.ndarray, n: int) -> np.ndarray:
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        out = np.zeros(n, dtype=np.float32)
        self.lib.oracle_dequant_q4k(_ptr(raw, _c_u8p), _ptr(out, _c_f32p), n)
        return out

    def dequant(self, type_: int, raw: np.ndarray, rows: int, n: int) -> np.ndarray:
        """rows x n weights of any fh3_dequant type -> fp32 [rows][n]."""
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        rb = self.row_bytes(type_, n)
        out = np.zeros((rows, n), dtype=np.float32)
        for r in range(rows):
            row = np.ascontiguousarray(raw[r * rb:(r + 1) * rb])
            rc = self.lib.oracle_dequant(type_, _ptr(row, _c_u8p), _ptr(out[r], _c_f32p), n)
            if rc != 0:
                raise ValueError(f"oracle_dequant: type {type_} not supported")
        return out

    def dequant_rows(self, raw: np.ndarray, rows: int, n: int) -> np.ndarray:
        rb = self.row_bytes(Q4K, n)
        raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(rows, rb)
        return np.stack([self.dequant_q4k(raw[r], n) for r in range(rows)])

    def matmul(self, type_: int, w: np.ndarray, in_: int, out: int, x: np.ndarray,
               bias: np.ndarray | None = None) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        n_tok = x.shape[0]
        y = np.empty((n_tok, out), dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        rc = self.lib.oracle_matmul(type_, _ptr(w, _c_u8p), in_, out, _ptr(x, _c_f32p),
                                    _ptr(y, _c_f32p), n_tok, _ptr(b, _c_f32p))
        if rc != 0:
            raise ValueError(f"oracle_matmul rejected its arguments (rc={rc})")
        return y

    def swiglu(self, h: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(h, dtype=np.float32)
        n, two_f = h.shape
        out = np.empty((n, two_f // 2), dtype=np.float32)
        self.lib.oracle_swiglu(_ptr(h, _c_f32p), _ptr(out, _c_f32p), n, two_f // 2)
        return out

    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        w = np.ascontiguousarray(w, dtype=np.float32)
        self.lib.oracle_rmsnorm(_ptr(x, _c_f32p), _ptr(w, _c_f32p), x.shape[0], x.shape[1], eps)
        return x

    def rope3(self, x: np.ndarray, cos: np.ndarray, sin: np.ndarray, heads: int, head_dim: int,
              rot_dim: int) -> np.ndarray:
        """x [n][heads*head_dim] rotated per head (a copy); cos/sin [n][rot_dim]."""
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        c = np.ascontiguousarray(cos, dtype=np.float32)
        s = np.ascontiguousarray(sin, dtype=np.float32)
        self.lib.oracle_rope3(_ptr(x, _c_f32p), _ptr(c, _c_f32p), _ptr(s, _c_f32p), x.shape[0], heads,
                              head_dim, rot_dim)
        return x

    def attention(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, heads: int, hd: int) -> np.ndarray:
        """q/k/v [n][heads*hd] fp32 -> o [n][heads*hd] (fh3_attention semantics)."""
        q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
        o = np.empty_like(q)
        self.lib.oracle_attention(_ptr(q, _c_f32p), _ptr(k, _c_f32p), _ptr(v, _c_f32p), _ptr(o, _c_f32p),
                                  q.shape[0], heads, hd)
        return o

    def vsa_tiles(self, seq: tuple, tile: int = 64) -> tuple[int, int, int]:
        """(num_tiles, num_prefix_tiles, num_video_tiles) of seq = (n, T, A, V, gt, gh, gw)."""
        out = (ctypes.c_int * 3)()
        if self.lib.oracle_vsa_tiles(*seq, tile, out):
            raise ValueError("empty sequence")
        return out[0], out[1], out[2]

    def vsa(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, gate: np.ndarray | None, seq: tuple, heads: int,
            hd: int, tile: int = 64, sparsity: float = 0.8, want_tiles: bool = False):
        """fh3_vsa_attention semantics; q/k/v/gate [n][heads*hd] fp32, seq = (n, T, A, V, gt, gh, gw).
        With want_tiles also returns the tile scores and the 0/1 tile mask, [heads][nt][nt]."""
        q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
        g = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32)
        o = np.zeros_like(q)
        nt = self.vsa_tiles(seq, tile)[0]
        sc = np.zeros((heads, nt, nt), np.float32) if want_tiles else None
        mk = np.zeros((heads, nt, nt), np.uint8) if want_tiles else None
        rc = self.lib.oracle_vsa(tile, sparsity, _ptr(q, _c_f32p), _ptr(k, _c_f32p), _ptr(v, _c_f32p),
                                 _ptr(g, _c_f32p), _ptr(o, _c_f32p), *seq, heads, hd, _ptr(sc, _c_f32p),
                                 _ptr(mk, _c_u8p))
        if rc:
            raise ValueError(f"oracle_vsa failed ({rc})")
        return (o, sc, mk) if want_tiles else o

    def qk_norm_rope(self, x: np.ndarray, w: np.ndarray, cos: np.ndarray, sin: np.ndarray, heads: int,
                     head_dim: int, rot_dim: int, eps: float) -> np.ndarray:
        """fh3_dit.c:397-401 for one of q / k: per-head rmsnorm, then rope3 (a copy)."""
        n = x.shape[0]
        y = self.rmsnorm(np.asarray(x, dtype=np.float32).reshape(n * heads, head_dim), w, eps)
        y = y.reshape(n, heads * head_dim)
        return self.rope3(y, cos, sin, heads, head_dim, rot_dim) if rot_dim > 0 else y

    def modulate(self, x: np.ndarray, shift: np.ndarray, scale: np.ndarray) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        sh = np.ascontiguousarray(np.broadcast_to(shift, x.shape), dtype=np.float32)
        sc = np.ascontiguousarray(np.broadcast_to(scale, x.shape), dtype=np.float32)
        self.lib.oracle_modulate(_ptr(x, _c_f32p), _ptr(sh, _c_f32p), _ptr(sc, _c_f32p),
                                 x.shape[0], x.shape[1])
        return x

    def gate_residual(self, h: np.ndarray, gate: np.ndarray, y: np.ndarray) -> np.ndarray:
        h = np.array(h, dtype=np.float32, copy=True, order="C")
        g = np.ascontiguousarray(np.broadcast_to(gate, h.shape), dtype=np.float32)
        y = np.ascontiguousarray(y, dtype=np.float32)
        self.lib.oracle_gate_residual(_ptr(h, _c_f32p), _ptr(g, _c_f32p), _ptr(y, _c_f32p),
                                      h.shape[0], h.shape[1])
        return h

    def rng_normal(self, seed: int, stream: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.lib.oracle_rng_normal(seed, stream, _ptr(out, _c_f32p), n)
        return out

    def quantize_q4k(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, n = x.shape
        out = np.empty(rows * self.row_bytes(Q4K, n), dtype=np.uint8)
        rc = self.lib.oracle_quantize_q4k(_ptr(x, _c_f32p), _ptr(out, _c_u8p), rows, n)
        if rc != 0:
            raise ValueError("oracle_quantize_q4k: n must be a positive multiple of 256")
        return out

    def make_weights(self, seed: int, stream: int, rows: int, n: int, scale: float = 0.02,
                     out: np.ndarray | None = None) -> np.ndarray:
        """Seeded Q4_K weights: quantise(scale * fh3_rng_normal(seed, stream))."""
        nbytes = rows * self.row_bytes(Q4K, n)
        if out is None:
            out = np.empty(nbytes, dtype=np.uint8)
        assert out.nbytes >= nbytes and out.dtype == np.uint8 and out.flags.c_contiguous
        rc = self.lib.oracle_make_q4k_weights(seed, stream, scale, rows, n, _ptr(out, _c_u8p))
        if rc != 0:
            raise ValueError(f"oracle_make_q4k_weights failed (rc={rc})")
        return out

    def num_threads(self) -> int:
        return int(self.lib.oracle_num_threads())


class Reference:
    """The reference's own functions, compiled from its sources into _ref/."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = ctypes.CDLL(path)
        lib.fh3_row_bytes.restype = ctypes.c_size_t
        lib.fh3_row_bytes.argtypes = [ctypes.c_int, ctypes.c_int64]
        lib.fh3_dequant.argtypes = [ctypes.c_int, ctypes.c_void_p, _c_f32p, ctypes.c_int64]
        for name in ("fh3_matmul", "fh3_matmul_scalar", "fh3_matmul_avx2"):
            f = getattr(lib, name)
            f.argtypes = [ctypes.POINTER(_Fh3W), _c_f32p, _c_f32p, ctypes.c_int, _c_f32p]
        lib.fh3_swiglu.argtypes = [_c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int]
        lib.fh3_rmsnorm.argtypes = [_c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        lib.fh3_modulate.argtypes = [_c_f32p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int]
        lib.fh3_rope3.argtypes = [_c_f32p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int]
        lib.fh3_attention.argtypes = [_c_f32p, _c_f32p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int]
        lib.fh3_gate_residual.argtypes = [_c_f32p, _c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int]
        lib.fh3_rng_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, _c_f32p, ctypes.c_size_t]
        lib.fh3_vsa_attention.argtypes = [ctypes.POINTER(_Fh3VsaCfg)] + [_c_f32p] * 5 + [
            ctypes.POINTER(_Fh3Seq), ctypes.c_int, ctypes.c_int]
        lib.fh3_seq_build.restype = ctypes.c_int
        lib.fh3_seq_build.argtypes = [ctypes.POINTER(_Fh3SeqSpec), ctypes.POINTER(_Fh3Seq)]
        lib.fh3_seq_free.argtypes = [ctypes.POINTER(_Fh3Seq)]
        self.lib = lib

    @staticmethod
    def available(path: str = REF_SO) -> bool:
        return os.path.exists(path)

    def row_bytes(self, type_: int, n: int) -> int:
        return int(self.lib.fh3_row_bytes(type_, n))

    def dequant(self, type_: int, raw: np.ndarray, n: int) -> np.ndarray:
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        out = np.zeros(n, dtype=np.float32)
        self.lib.fh3_dequant(type_, raw.ctypes.data, _ptr(out, _c_f32p), n)
        return out

    def matmul(self, type_: int, w: np.ndarray, in_: int, out: int, x: np.ndarray,
               bias: np.ndarray | None = None, variant: str = "fh3_matmul") -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros((x.shape[0], out), dtype=np.float32)
        desc = _Fh3W(type_, in_, out, _ptr(w, _c_u8p))
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        getattr(self.lib, variant)(ctypes.byref(desc), _ptr(x, _c_f32p), _ptr(y, _c_f32p),
                                   x.shape[0], _ptr(b, _c_f32p))
        return y

    def matmul_into(self, desc: "_Fh3W", x: np.ndarray, y: np.ndarray, n_tok: int,
                    bias: np.ndarray | None = None) -> None:
        """Unchecked call used by the timed CPU baseline (buffers preallocated)."""
        self.lib.fh3_matmul(ctypes.byref(desc), _ptr(x, _c_f32p), _ptr(y, _c_f32p), n_tok,
                            _ptr(bias, _c_f32p) if bias is not None else None)

    def swiglu(self, h: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(h, dtype=np.float32)
        n, two_f = h.shape
        out = np.empty((n, two_f // 2), dtype=np.float32)
        self.lib.fh3_swiglu(_ptr(h, _c_f32p), _ptr(out, _c_f32p), n, two_f // 2)
        return out

    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        w = np.ascontiguousarray(w, dtype=np.float32)
        self.lib.fh3_rmsnorm(_ptr(x, _c_f32p), _ptr(w, _c_f32p), x.shape[0], x.shape[1], eps)
        return x

    def attention(self, q, k, v, heads: int, hd: int):
        q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
        o = np.empty_like(q)
        self.lib.fh3_attention(_ptr(q, _c_f32p), _ptr(k, _c_f32p), _ptr(v, _c_f32p), _ptr(o, _c_f32p),
                               q.shape[0], heads, hd)
        return o

    def seq_build(self, num_text: int, num_audio: int, num_video: int, pos: np.ndarray | None = None, **spec):
        """fh3_seq_build itself: (pair_index [N], cos [N][96], sin [N][96]) of a sequence."""
        p = None if pos is None else np.ascontiguousarray(pos, dtype=np.float64)
        sp = _Fh3SeqSpec(num_text=num_text, num_audio=num_audio, num_video=num_video,
                         custom_pos=None if p is None else p.ctypes.data, **spec)
        sq = _Fh3Seq()
        if self.lib.fh3_seq_build(ctypes.byref(sp), ctypes.byref(sq)):
            raise ValueError("fh3_seq_build failed")
        n = sq.seq_len
        pair = np.ctypeslib.as_array(ctypes.cast(sq.pair_index, ctypes.POINTER(ctypes.c_int)), (n,)).copy()
        cos = np.ctypeslib.as_array(ctypes.cast(sq.cos, _c_f32p), (n, 96)).copy()
        sin = np.ctypeslib.as_array(ctypes.cast(sq.sin, _c_f32p), (n, 96)).copy()
        self.lib.fh3_seq_free(ctypes.byref(sq))
        return pair, cos, sin

    def vsa(self, q, k, v, gate, seq: tuple, heads: int, hd: int, tile: int = 64, sparsity: float = 0.8):
        """fh3_vsa_attention itself; seq = (n, T, A, V, gt, gh, gw)."""
        q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
        g = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32)
        o = np.zeros_like(q)
        sq = _Fh3Seq(*seq)
        cfg = _Fh3VsaCfg(tile, sparsity)
        self.lib.fh3_vsa_attention(ctypes.byref(cfg), _ptr(q, _c_f32p), _ptr(k, _c_f32p), _ptr(v, _c_f32p),
                                   _ptr(g, _c_f32p), _ptr(o, _c_f32p), ctypes.byref(sq), heads, hd)
        return o

    def rope3(self, x, cos, sin, heads: int, head_dim: int, rot_dim: int):
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        c = np.ascontiguousarray(cos, dtype=np.float32)
        s = np.ascontiguousarray(sin, dtype=np.float32)
        self.lib.fh3_rope3(_ptr(x, _c_f32p), _ptr(c, _c_f32p), _ptr(s, _c_f32p), x.shape[0], heads, head_dim,
                           rot_dim)
        return x

    def modulate(self, x, shift, scale):
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        sh = np.ascontiguousarray(np.broadcast_to(shift, x.shape), dtype=np.float32)
        sc = np.ascontiguousarray(np.broadcast_to(scale, x.shape), dtype=np.float32)
        self.lib.fh3_modulate(_ptr(x, _c_f32p), _ptr(sh, _c_f32p), _ptr(sc, _c_f32p),
                              x.shape[0], x.shape[1])
        return x

    def gate_residual(self, h, gate, y):
        h = np.array(h, dtype=np.float32, copy=True, order="C")
        g = np.ascontiguousarray(np.broadcast_to(gate, h.shape), dtype=np.float32)
        y = np.ascontiguousarray(y, dtype=np.float32)
        self.lib.fh3_gate_residual(_ptr(h, _c_f32p), _ptr(g, _c_f32p), _ptr(y, _c_f32p),
                                   h.shape[0], h.shape[1])
        return h

    def rng_normal(self, seed: int, stream: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.lib.fh3_rng_normal(seed, stream, _ptr(out, _c_f32p), n)
        return out


def rel_fro(a: np.ndarray, b: np.ndarray) -> float:
    """Relative Frobenius error ||a-b|| / ||b|| in float64."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
