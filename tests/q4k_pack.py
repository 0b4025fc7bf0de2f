"""Test infrastructure for the DiT forward on a Q4_K trunk: an FH3P rewriter and the oracle's
composition of fh3_dit_forward.

* write_q4k_pack: reads a packed trunk (FH3P, the layout of src/io/fh3_pack.h:29-88) and writes
  a copy whose projections (qkv, gate_compress, out, fc1, fc2) are quantised to Q4_K by the
  oracle's quantiser, norm weights kept F32 -- a synthetic Q4_K pack in the layout the
  reference's packer writes.
* oracle_forward: fh3_dit_forward (src/model/fh3_dit.c:340-467) composed from the oracle's
  restatements of fh3_rmsnorm, fh3_modulate, fh3_matmul, fh3_rope3, fh3_attention,
  fh3_vsa_attention, fh3_swiglu and fh3_gate_residual, all in fp32 on the CPU.
"""
from __future__ import annotations

import struct

import numpy as np

PACK_MAGIC, ADALN_MAGIC = 0x50334846, 0x41334846
TENSORS = ("qkv", "gate_compress", "out", "fc1", "fc2", "norm1", "norm2", "q_norm", "k_norm")
PROJECTIONS = ("qkv", "gate_compress", "out", "fc1", "fc2")
DESC, TDESC, ALIGN = 24, 168, 4096


def read_pack(path: str):
    """[(layer tensors {name: dict(type, in, out, raw bytes, desc bytes)})] of an FH3P file."""
    b = open(path, "rb").read()
    magic, ver, nl, align = struct.unpack_from("<IIII", b, 0)
    assert magic == PACK_MAGIC and ver == 1 and align == ALIGN
    index_off, index_bytes = struct.unpack_from("<QQ", b, 16)
    stride = index_bytes // nl
    layers = []
    for L in range(nl):
        d = index_off + L * stride
        foff, size, nt = struct.unpack_from("<QQI", b, d)
        ts = {}
        for t in range(nt):
            td = d + DESC + t * TDESC
            typ = struct.unpack_from("<I", b, td + 64)[0]
            off, sz, ind, outd = struct.unpack_from("<QQqq", b, td + 104)
            name = TENSORS[t] if t < len(TENSORS) else f"extra{t}"
            ts[name] = dict(type=typ, in_=ind, out=outd, raw=np.frombuffer(b, np.uint8, sz, foff + off).copy(),
                            desc=bytearray(b[td:td + TDESC]))
        layers.append(ts)
    return layers


def write_q4k_pack(src: str, dst: str, oracle) -> list:
    """Copy of the FH3P file src with its F32 projections quantised to Q4_K; returns the layers."""
    layers = read_pack(src)
    for ts in layers:
        for name in PROJECTIONS:
            t = ts.get(name)
            if t is None or t["type"] != 0 or t["out"] <= 0 or t["in_"] % 256:
                continue
            w = t["raw"].view(np.float32).reshape(t["out"], t["in_"])
            t["raw"] = oracle.quantize_q4k(w)
            t["type"] = 12
    nl = len(layers)
    nt = max(len(ts) for ts in layers)
    stride = DESC + nt * TDESC
    index_off = 128
    data_off = (index_off + nl * stride + ALIGN - 1) // ALIGN * ALIGN
    runs, pos = [], data_off
    for ts in layers:
        off, placed = 0, []
        for name in list(TENSORS) + [k for k in ts if k not in TENSORS]:
            if name not in ts:
                continue
            placed.append((name, off))
            off += (len(ts[name]["raw"]) + 255) // 256 * 256
        runs.append((pos, off, placed))
        pos += (off + ALIGN - 1) // ALIGN * ALIGN
    out = bytearray(pos)
    struct.pack_into("<IIIIQQQQ", out, 0, PACK_MAGIC, 1, nl, ALIGN, index_off, nl * stride, data_off, pos)
    for L, (ts, (foff, size, placed)) in enumerate(zip(layers, runs)):
        d = index_off + L * stride
        struct.pack_into("<QQII", out, d, foff, size, len(placed), 0)
        for t, (name, off) in enumerate(placed):
            x = ts[name]
            desc = bytearray(x["desc"])
            struct.pack_into("<I", desc, 64, x["type"])
            struct.pack_into("<QQ", desc, 104, off, len(x["raw"]))
            out[d + DESC + t * TDESC:d + DESC + (t + 1) * TDESC] = desc
            out[foff + off:foff + off + len(x["raw"])] = x["raw"].tobytes()
    with open(dst, "wb") as f:
        f.write(out)
    return layers


def read_adaln(path: str):
    """(trunk [steps][blocks][pairs][6][hidden], final [steps][pairs][2][hidden] or None) of an FH3A file."""
    b = open(path, "rb").read()
    magic, ver, ns, nb, pairs, hid = struct.unpack_from("<IIIIII", b, 0)
    assert magic == ADALN_MAGIC and ver == 1
    toff, tbytes, foff, fbytes = struct.unpack_from("<QQQQ", b, 32)
    trunk = np.frombuffer(b, np.float32, ns * nb * pairs * 6 * hid, toff).reshape(ns, nb, pairs, 6, hid)
    fin = np.frombuffer(b, np.float32, ns * pairs * 2 * hid, foff).reshape(ns, pairs, 2, hid) if fbytes else None
    return trunk, fin


def _mat(oracle, t, x):
    return oracle.matmul(t["type"], t["raw"], t["in_"], t["out"], x)


def oracle_forward(oracle, layers, glob: dict, adaln, text_rows, x_video, x_audio, cos, sin, step: int, cfg: dict,
                   seq: tuple):
    """fh3_dit_forward in fp32 on the CPU.  glob maps the globals' names to fp32 arrays; rows are
    text | audio | video with AdaLN pairs 1, 2, 0; cfg: hidden, heads, head_dim, ffn, eps, qk_eps,
    final_eps, attn (0 dense, 1 video sparse), vsa_tile, vsa_sparsity."""
    trunk, fin = adaln
    T, A, V = len(text_rows), len(x_audio), len(x_video)
    N, hid, heads, hd = T + A + V, cfg["hidden"], cfg["heads"], cfg["head_dim"]
    inner = heads * hd
    pair = np.array([1] * T + [2] * A + [0] * V)

    def rows_of(L, chunk):
        tab = trunk[step, L] if L >= 0 else fin[step]
        return tab[pair, chunk]                      # [N][hid]

    def lin(name, x):
        w = glob[name + ".weight"]
        y = oracle.matmul(0, np.ascontiguousarray(w, np.float32).view(np.uint8), w.shape[1], w.shape[0], x)
        b = glob.get(name + ".bias")
        return y + b[None, :] if b is not None else y

    h = np.concatenate([text_rows, lin("audio_patch_proj", x_audio), lin("video_patch_proj", x_video)]).astype(np.float32)
    for L, ts in enumerate(layers):
        nw1 = ts["norm1"]["raw"].view(np.float32)
        nw2 = ts["norm2"]["raw"].view(np.float32)
        normed = oracle.modulate(oracle.rmsnorm(h, nw1, cfg["eps"]), rows_of(L, 0), rows_of(L, 1))
        qkv = _mat(oracle, ts["qkv"], normed)
        q = oracle.qk_norm_rope(qkv[:, :inner], ts["q_norm"]["raw"].view(np.float32), cos, sin, heads, hd, 96,
                                cfg["qk_eps"])
        k = oracle.qk_norm_rope(qkv[:, inner:2 * inner], ts["k_norm"]["raw"].view(np.float32), cos, sin, heads, hd,
                                96, cfg["qk_eps"])
        v = np.ascontiguousarray(qkv[:, 2 * inner:])
        if cfg["attn"] == 1:
            g = ts.get("gate_compress")
            gate = _mat(oracle, g, normed) if g is not None and g["out"] > 0 else None
            att = oracle.vsa(q, k, v, gate, seq, heads, hd, cfg["vsa_tile"], cfg["vsa_sparsity"])
        else:
            att = oracle.attention(q, k, v, heads, hd)
        h = oracle.gate_residual(h, rows_of(L, 2), _mat(oracle, ts["out"], att))
        normed = oracle.modulate(oracle.rmsnorm(h, nw2, cfg["eps"]), rows_of(L, 3), rows_of(L, 4))
        h = oracle.gate_residual(h, rows_of(L, 5), _mat(oracle, ts["fc2"], oracle.swiglu(_mat(oracle, ts["fc1"], normed))))
    normed = oracle.modulate(oracle.rmsnorm(h, glob["final_layer.norm.weight"], cfg["final_eps"]), rows_of(-1, 0),
                             rows_of(-1, 1))
    return lin("final_layer.video_out", normed[T + A:]), lin("final_layer.audio_out", normed[T:T + A])
