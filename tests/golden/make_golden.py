"""Regenerate the golden vectors under tests/golden/ (run in a tree that has the reference).

1. Copies the reference's own Q4_K golden vectors (data files, not sources):
     tests/fixtures/quant/Q4_K.bin        -> Q4_K.bin        (gguf-py dequantize output)
     tests/fixtures/quant/matmul_ref.bin  -> matmul_ref.bin  (fp64 numpy matmul output)
   Their layouts are documented in the reference's tools/emit_quant_fixtures.py:75-81,134-141
   and read by tests/unit/test_quant.c:54-81 and tests/unit/test_matmul.c:196-231.
   The other formats' fixtures tests/fixtures/quant/{F16,BF16,Q8_0,Q2_K,Q3_K,Q5_K,Q6_K}.bin (same
   layout as Q4_K.bin: <u32 type, rows, cols, nbytes>, raw bytes, gguf-py's fp32 dequantisation).
   Also the op fixtures tests/fixtures/ops/{rmsnorm,rope3}.bin -> {rmsnorm,rope3}.bin,
   read by the reference's tests/unit/test_ops.c:58-96 (<u32 n, u32 dim, f32 eps>, x, w, ref)
   and :98-140 (<u32 n, heads, head_dim, rot_dim>, x, cos, sin, ref).
   And the video-sparse-attention fixtures tests/fixtures/vsa/{vsa_n784,vsa_padded,vsa_sparsity0}.bin
   -> vsa/*.bin (<u32 n, T, A, V, grid_t, grid_h, grid_w, heads, head_dim; f32 sparsity; u32 has_gate>,
   then q, k, v, [gate], ref as [n][heads][head_dim] fp32), read by tests/unit/test_vsa.c:56-133.
   And the tiny end-to-end model tests/fixtures/tiny_h3/ -> tiny_h3/ (tools/make_tiny_h3.py: a
   3-layer F32 DiT packed as FH3P + FH3A + GGUF globals, inputs, and torch's outputs at steps 0 and 7,
   dense and VSA), read by tests/unit/test_dit_tiny.c.
2. Writes ref_cases.npz: seeded inputs (this project's Q4_K quantiser + fh3_rng_normal)
   with outputs computed by the REFERENCE'S OWN fh3_matmul / fh3_dequant / fh3_swiglu,
   compiled from its sources into oracle/_ref/libfh3ref.so (oracle/Makefile).  These pin
   the oracle and the CUDA path on shapes the reference's goldens do not cover
   (odd N, tiny K, GEMV token counts, a GEMM-sized M).

    python tests/golden/make_golden.py [--ref /path/to/fh3]
"""
from __future__ import annotations

import argparse
import os
import shutil
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import Q4K, Oracle, Reference, build  # noqa: E402

# (name, K, N, M, bias?)  -- seeds are derived from the index
CASES = [
    ("k256_n1_m1", 256, 1, 1, False),
    ("k512_n70_m1", 512, 70, 1, True),
    ("k512_n70_m3", 512, 70, 3, False),
    ("k1024_n130_m16", 1024, 130, 16, True),
    ("k768_n200_m5", 768, 200, 5, False),
    ("k1024_n192_m37", 1024, 192, 37, True),
    ("k512_n264_m130", 512, 264, 130, True),
]


TINY_H3 = ("meta.json", "dit_trunk.bin", "dit_globals.bin", "adaln_table.bin", "pos.bin", "x_video.bin",
           "x_audio.bin", "text_emb.bin", "text_rows.bin", "video_v_step0.bin", "video_v_step7.bin",
           "audio_v_step0.bin", "audio_v_step7.bin", "video_v_vsa_step0.bin", "video_v_vsa_step7.bin",
           "audio_v_vsa_step0.bin", "audio_v_vsa_step7.bin")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="the reference source tree (default: $FH3_REF_TREE or "
                                                 "BASELINE.json's reference_path)")
    args = ap.parse_args()
    if args.ref is None:
        sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
        from oracle.oracle import reference_tree
        args.ref = reference_tree()
    if not args.ref:
        raise SystemExit("the reference source tree was not found: pass --ref or set FH3_REF_TREE")
    fx = os.path.join(args.ref, "tests", "fixtures", "quant")
    for name in ("Q4_K.bin", "matmul_ref.bin", "F16.bin", "BF16.bin", "Q8_0.bin", "Q2_K.bin", "Q3_K.bin",
                 "Q5_K.bin", "Q6_K.bin"):
        shutil.copyfile(os.path.join(fx, name), os.path.join(HERE, name))
    for name in ("rmsnorm.bin", "rope3.bin"):
        shutil.copyfile(os.path.join(args.ref, "tests", "fixtures", "ops", name), os.path.join(HERE, name))
    os.makedirs(os.path.join(HERE, "vsa"), exist_ok=True)
    for name in ("vsa_n784.bin", "vsa_padded.bin", "vsa_sparsity0.bin"):
        shutil.copyfile(os.path.join(args.ref, "tests", "fixtures", "vsa", name), os.path.join(HERE, "vsa", name))
    os.makedirs(os.path.join(HERE, "tiny_h3"), exist_ok=True)
    for name in TINY_H3:
        shutil.copyfile(os.path.join(args.ref, "tests", "fixtures", "tiny_h3", name), os.path.join(HERE, "tiny_h3", name))
    build()
    o = Oracle()
    r = Reference()
    out = {}
    for i, (name, K, N, M, has_bias) in enumerate(CASES):
        w = o.make_weights(seed=1000 + i, stream=1, rows=N, n=K)
        x = o.rng_normal(1000 + i, 2, M * K).reshape(M, K)
        b = o.rng_normal(1000 + i, 3, N) if has_bias else None
        y = r.matmul(Q4K, w, K, N, x, b)
        out[f"{name}/w"] = w
        out[f"{name}/x"] = x
        if b is not None:
            out[f"{name}/bias"] = b
        out[f"{name}/y"] = y
        out[f"{name}/dims"] = np.array([K, N, M], dtype=np.int64)
    # dequant of one generated matrix, by the reference
    w = o.make_weights(seed=77, stream=5, rows=3, n=1024)
    out["dequant/w"] = w
    out["dequant/y"] = np.stack([r.dequant(Q4K, w[i * 576:(i + 1) * 576], 1024) for i in range(3)])
    # swiglu by the reference
    h = (o.rng_normal(78, 1, 4 * 2 * 96) * 4.0).reshape(4, 192)
    h[0, 96:100] = [-100.0, -80.5, -79.5, 90.0]
    out["swiglu/h"] = h
    out["swiglu/y"] = r.swiglu(h)
    # q/k normalisation + rope as fh3_dit.c:397-401 (40 heads x 128, rot 96), by the reference
    n, H, D, R = 7, 40, 128, 96
    x = (o.rng_normal(79, 1, n * H * D) * 3.0).reshape(n, H * D)
    wq = 1.0 + 0.1 * o.rng_normal(79, 2, D)
    ang = o.rng_normal(79, 3, n * R).reshape(n, R)
    cs, sn = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    out["qkrope/x"], out["qkrope/w"], out["qkrope/cos"], out["qkrope/sin"] = x, wq, cs, sn
    out["qkrope/dims"] = np.array([n, H, D, R], dtype=np.int64)
    out["qkrope/y"] = r.rope3(r.rmsnorm(x.reshape(n * H, D), wq, 1e-6).reshape(n, H * D), cs, sn, H, D, R)
    # dense attention (fh3_attention), by the reference: n not a multiple of the 64-key tile
    n, H, D = 200, 2, 128
    for nm, st in (("q", 1), ("k", 2), ("v", 3)):
        out[f"attn/{nm}"] = o.rng_normal(80, st, n * H * D).reshape(n, H * D)
    out["attn/dims"] = np.array([n, H, D], dtype=np.int64)
    out["attn/y"] = r.attention(out["attn/q"], out["attn/k"], out["attn/v"], H, D)
    # fh3_matmul on the other formats' fixture weights (rows x 512), by the reference
    import struct
    for i, nm in enumerate(("F16", "BF16", "Q8_0", "Q2_K", "Q3_K", "Q5_K", "Q6_K")):
        with open(os.path.join(HERE, f"{nm}.bin"), "rb") as f:
            b = f.read()
        t, rows, cols, nb = struct.unpack("<IIII", b[:16])
        w = np.frombuffer(b[16:16 + nb], np.uint8).copy()
        x = o.rng_normal(90 + i, 1, 5 * cols).reshape(5, cols)
        bias = o.rng_normal(90 + i, 2, rows)
        out[f"fmt_{nm}/w"] = w
        out[f"fmt_{nm}/x"] = x
        out[f"fmt_{nm}/bias"] = bias
        out[f"fmt_{nm}/dims"] = np.array([t, cols, rows, 5], dtype=np.int64)
        out[f"fmt_{nm}/y"] = r.matmul(t, w, cols, rows, x, bias)
    # fh3_vsa_attention by the reference on cases its fixtures do not cover:
    # (name, seq = (n, T, A, V, gt, gh, gw), heads, head_dim, tile, sparsity, gate?, tied video key tiles?)
    vsa_cases = [
        ("hd128_tied", (8 + 4 * 4 * 16, 8, 0, 256, 4, 4, 16), 1, 128, 64, 0.6, True, True),
        ("nogate_tile32", (40 + 30 + 4 * 5 * 6, 40, 30, 120, 4, 5, 6), 2, 64, 32, 0.7, False, False),
        ("tile100", (130 + 128, 130, 0, 128, 4, 4, 8), 1, 64, 100, 0.9, True, False),
        ("mismatch_allvideo", (200, 50, 50, 50, 2, 5, 5), 1, 64, 64, 0.5, True, False),
        ("badgrid", (20 + 150, 20, 0, 150, 3, 7, 7), 1, 64, 64, 0.6, True, False),
    ]
    for ci, (nm, seq, H, D, tile, sp, has_gate, tied) in enumerate(vsa_cases):
        n = seq[0]
        qv = o.rng_normal(120 + ci, 1, n * H * D).reshape(n, H * D)
        kv = o.rng_normal(120 + ci, 2, n * H * D).reshape(n, H * D)
        vv = o.rng_normal(120 + ci, 3, n * H * D).reshape(n, H * D)
        gv = o.rng_normal(120 + ci, 4, n * H * D).reshape(n, H * D) if has_gate else None
        if tied:  # every video token's k equal to the first video token's: all video tile scores tie
            kv[seq[1] + seq[2]:] = kv[seq[1] + seq[2]]
        out[f"vsa_{nm}/q"], out[f"vsa_{nm}/k"], out[f"vsa_{nm}/v"] = qv, kv, vv
        if gv is not None:
            out[f"vsa_{nm}/gate"] = gv
        out[f"vsa_{nm}/seq"] = np.array(seq, dtype=np.int64)
        out[f"vsa_{nm}/cfg"] = np.array([H, D, tile], dtype=np.int64)
        out[f"vsa_{nm}/sparsity"] = np.array([sp], dtype=np.float32)
        out[f"vsa_{nm}/y"] = r.vsa(qv, kv, vv, gv, seq, H, D, tile, sp)
    # fh3_rng_normal itself
    out["rng/seed7_stream3"] = r.rng_normal(7, 3, 1001)
    np.savez_compressed(os.path.join(HERE, "ref_cases.npz"), **out)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
