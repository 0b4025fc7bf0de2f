"""The DiT forward of fh3 on the GPU, host side: the model layer above libfh3cuda.

Mirrors fh3's src/model API (fh3_dit_open / fh3_dit_prepare_text / fh3_dit_forward,
src/model/fh3_dit.c) with the I/O of src/io replaced by one-time uploads to HBM:

* ``Pack``    -- the packed trunk (FH3P), ``fh3cuda_pack_open`` (replaces the NVMe ring);
* ``Adaln``   -- the folded AdaLN table (FH3A), ``fh3cuda_adaln_open``;
* ``read_gguf`` -- the globals file (GGUF v2/v3: patch / condition projections, text
  refiner, final layer), read here as fh3_gguf.c reads it, uploaded by ``DitGlobals``;
* ``rope_tables`` -- the [N][96] cos / sin tables of fh3_seq_build (src/model/fh3_seq.c:147-168);
* ``Dit``     -- ``prepare_text`` and ``forward`` through fh3cuda_dit_prepare_text_dev /
  fh3cuda_dit_forward_dev (all compute on the device).
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass

import numpy as np

from . import F32, _ensure, _ptr, _stream, _torch, check, dequant, load, row_bytes
from ._lib import (Fh3CudaDitCfg, Fh3CudaDitGlobals, Fh3CudaLayerView, Fh3CudaSeq, Fh3CudaW)

ATTN_DENSE, ATTN_VSA = 0, 1   # fh3's Fh3AttnType (include/fh3/fh3.h:37-40)

# GGUF metadata value types and their struct codes (fixed-size ones)
_GGUF_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
_GGUF_STRING, _GGUF_ARRAY = 8, 9


@dataclass
class GgufTensor:
    name: str
    type: int
    ne: tuple            # ne[0] innermost (the "in" dimension of a weight)
    offset: int          # from the start of the data section


class _Reader:
    def __init__(self, buf: bytes):
        self.b, self.o = buf, 0

    def take(self, fmt: str):
        v = struct.unpack_from("<" + fmt, self.b, self.o)
        self.o += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string(self) -> str:
        n = self.take("Q")
        s = self.b[self.o:self.o + n].decode("utf-8", errors="replace")
        self.o += n
        return s

    def value(self, t: int):
        if t in _GGUF_SCALAR:
            return self.take(_GGUF_SCALAR[t])
        if t == _GGUF_STRING:
            return self.string()
        if t == _GGUF_ARRAY:
            et, n = self.take("I"), self.take("Q")
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"GGUF: unknown metadata type {t}")


def read_gguf(path: str):
    """(metadata dict, {name: GgufTensor}, raw file bytes, data section offset) of a GGUF file."""
    with open(path, "rb") as f:
        buf = f.read()
    r = _Reader(buf)
    magic, version = r.take("I"), r.take("I")
    if magic != 0x46554747:
        raise ValueError(f"{path}: not a GGUF file")
    if version not in (2, 3):
        raise ValueError(f"{path}: GGUF version {version}")
    n_tensors, n_kv = r.take("Q"), r.take("Q")
    meta = {}
    for _ in range(n_kv):
        key = r.string()
        meta[key] = r.value(r.take("I"))
    tensors = {}
    for _ in range(n_tensors):
        name = r.string()
        nd = r.take("I")
        ne = tuple(r.take("Q") for _ in range(nd))
        t, off = r.take("I"), r.take("Q")
        tensors[name] = GgufTensor(name, t, ne, off)
    align = int(meta.get("general.alignment", 32))
    data = (r.o + align - 1) // align * align
    return meta, tensors, buf, data


class Pack:
    """A packed DiT trunk (FH3P) resident in HBM (fh3cuda_pack_open)."""

    def __init__(self, path: str):
        self.h = ctypes.c_void_p()
        check(load().fh3cuda_pack_open(path.encode(), ctypes.byref(self.h)))

    @property
    def num_layers(self) -> int:
        return load().fh3cuda_pack_num_layers(self.h)

    @property
    def device_bytes(self) -> int:
        return int(load().fh3cuda_pack_device_bytes(self.h))

    def layer(self, L: int) -> Fh3CudaLayerView:
        v = Fh3CudaLayerView()
        check(load().fh3cuda_pack_layer(self.h, L, ctypes.byref(v)))
        return v

    def close(self) -> None:
        if self.h:
            load().fh3cuda_pack_close(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Adaln:
    """The folded AdaLN table (FH3A) resident in HBM (fh3cuda_adaln_open)."""

    def __init__(self, path: str, expect_hash: int = 0):
        self.h = ctypes.c_void_p()
        check(load().fh3cuda_adaln_open(path.encode(), expect_hash, ctypes.byref(self.h)))
        d = [ctypes.c_int() for _ in range(4)]
        check(load().fh3cuda_adaln_dims(self.h, *(ctypes.byref(x) for x in d)))
        self.n_steps, self.n_blocks, self.pairs, self.hidden = (x.value for x in d)

    def row(self, step: int, block: int, pair: int, chunk: int) -> int | None:
        """Device address of a row (fh3_adaln_row), None outside the table."""
        return load().fh3cuda_adaln_row(self.h, step, block, pair, chunk)

    def close(self) -> None:
        if self.h:
            load().fh3cuda_adaln_close(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DitGlobals:
    """The globals of fh3_dit_open (src/model/fh3_dit.c:55-180) uploaded to the device once."""

    def __init__(self, path: str, num_refiner_layers: int, device="cuda"):
        torch = _torch()
        _, tensors, buf, data = read_gguf(path)
        self.keep = []   # device tensors the struct points into
        g = Fh3CudaDitGlobals()

        def raw(t: GgufTensor):
            rows = int(np.prod(t.ne[1:])) if len(t.ne) > 1 else 1
            nb = rows * row_bytes(t.type, int(t.ne[0]))
            a = np.frombuffer(buf, np.uint8, nb, data + t.offset)
            d = torch.from_numpy(a.copy()).to(device)
            self.keep.append(d)
            return d, rows

        def weight(name: str, required: bool = True) -> Fh3CudaW:      # load_tensor_w (:43-53)
            t = tensors.get(name)
            if t is None:
                if required:
                    raise KeyError(f"{path}: tensor {name} missing")
                return Fh3CudaW()
            d, _ = raw(t)
            return Fh3CudaW(t.type, int(t.ne[0]), int(t.ne[1]) if len(t.ne) > 1 else 1, _ptr(d))

        def vec(name: str):                                                 # load_tensor_f32 (:12-41)
            t = tensors.get(name)
            if t is None:
                return None
            d, _ = raw(t)
            if t.type != F32:
                d = dequant(t.type, d, int(t.ne[0]))
                self.keep.append(d)
            return _ptr(d)

        g.video_patch_proj = weight("video_patch_proj.weight")
        g.video_patch_proj_bias = vec("video_patch_proj.bias")
        g.audio_patch_proj = weight("audio_patch_proj.weight")
        g.audio_patch_proj_bias = vec("audio_patch_proj.bias")
        g.condition_proj = weight("condition_proj.weight")
        g.condition_proj_bias = vec("condition_proj.bias")
        if not 0 <= num_refiner_layers <= 4:
            raise ValueError("num_refiner_layers must be 0..4")
        for r in range(num_refiner_layers):
            p = f"token_refiner.blocks.{r}."
            rb = g.refiner[r]
            rb.norm1 = vec(p + "norm1.weight")
            rb.qkv = weight(p + "attn.qkv_proj.weight", False)
            rb.q_norm = vec(p + "attn.q_norm.weight")
            rb.k_norm = vec(p + "attn.k_norm.weight")
            rb.out = weight(p + "attn.out_proj.weight", False)
            rb.norm2 = vec(p + "norm2.weight")
            rb.fc1 = weight(p + "mlp.fc1.weight", False)
            rb.fc2 = weight(p + "mlp.fc2.weight", False)
        g.refiner_final_norm = vec("token_refiner.final_norm.weight")
        g.final_norm = vec("final_layer.norm.weight")
        g.video_out = weight("final_layer.video_out.weight")
        g.video_out_bias = vec("final_layer.video_out.bias")
        g.audio_out = weight("final_layer.audio_out.weight")
        g.audio_out_bias = vec("final_layer.audio_out.bias")
        self.struct = g


def rope_tables(pos: np.ndarray):
    """cos, sin [N][96] fp32 of fh3_seq_build (src/model/fh3_seq.c:147-168) from positions
    pos [N][3] (t, h, w) fp64: 16 frequencies 1 / 10000^(k/16) per axis, angles rounded to
    fp32, channels [t h w t h w] x 16.  cos / sin of the fp32 angle are evaluated in fp64 and
    rounded once (within one ulp of the C library's cosf / sinf)."""
    pos = np.asarray(pos, dtype=np.float64).reshape(-1, 3)
    inv = 1.0 / np.power(10000.0, np.arange(16, dtype=np.float64) / 16.0)
    ang = (pos[:, :, None] * inv[None, None, :]).astype(np.float32)        # [N][3][16]
    ang = np.concatenate([ang[:, 0], ang[:, 1], ang[:, 2]] * 2, axis=1).astype(np.float64)   # [N][96]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class Dit:
    """fh3_dit_prepare_text / fh3_dit_forward on the device (fh3cuda_dit_*_dev)."""

    def __init__(self, cfg: Fh3CudaDitCfg, globals_: DitGlobals):
        self.cfg, self.g = cfg, globals_

    def prepare_text(self, text_emb, stream=None):
        torch = _torch()
        _ensure(text_emb)
        T = text_emb.shape[0]
        out = torch.empty((T, self.cfg.hidden_size), dtype=torch.float32, device=text_emb.device)
        check(load().fh3cuda_dit_prepare_text_dev(ctypes.byref(self.cfg), ctypes.byref(self.g.struct),
                                                  _ptr(text_emb.contiguous()), T, _ptr(out), _stream(stream)))
        return out

    def forward(self, trunk: Pack, adaln: Adaln, seq, cos, sin, step: int, x_video, x_audio, text_rows,
                stream=None):
        """seq = (N, T, A, V, grid_t, grid_h, grid_w); returns (v_video [V][video dim], v_audio [A][audio dim])."""
        torch = _torch()
        for t in (cos, sin, x_video, x_audio, text_rows):
            _ensure(t)
        V, A = seq[3], seq[2]
        vv = torch.empty((V, self.g.struct.video_out.out), dtype=torch.float32, device=x_video.device)
        va = torch.empty((A, self.g.struct.audio_out.out), dtype=torch.float32, device=x_video.device)
        check(load().fh3cuda_dit_forward_dev(
            ctypes.byref(self.cfg), ctypes.byref(self.g.struct), trunk.h, adaln.h, ctypes.byref(Fh3CudaSeq(*seq)),
            _ptr(cos.contiguous()), _ptr(sin.contiguous()), step, _ptr(x_video.contiguous()),
            _ptr(x_audio.contiguous()), _ptr(text_rows.contiguous()), _ptr(vv), _ptr(va), _stream(stream)))
        return vv, va
