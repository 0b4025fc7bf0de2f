"""Host side of the device DiT forward (fasth3inc_b200/dit.py, csrc/trunk_io.cu), no GPU needed.

* the GGUF reader against the reference's tiny globals file (35 F32 tensors) and, where gguf-py
  is importable, against gguf-py's own reading of it;
* the rope tables against the reference's fh3_seq_build (oracle/_ref): bit-exact on the tiny
  model's positions, within one ulp on random ones;
* the FH3P / FH3A readers' error codes, as fh3_pack_open / fh3_adaln_open return them
  (src/io/fh3_pack.c:23-60, :188-225); a well-formed file passes every file check and stops
  only at the missing device.
"""
from __future__ import annotations

import os
import struct

import numpy as np
import pytest

from conftest import GOLDEN, HAS_GPU

TINY = os.path.join(GOLDEN, "tiny_h3")


def test_gguf_reader_on_tiny_globals():
    from fasth3inc_b200.dit import read_gguf
    meta, tensors, buf, data = read_gguf(os.path.join(TINY, "dit_globals.bin"))
    assert len(tensors) == 35
    assert all(t.type == 0 for t in tensors.values())           # F32
    assert tensors["video_patch_proj.weight"].ne == (96, 256)
    assert tensors["token_refiner.blocks.1.mlp.fc1.weight"].ne == (256, 1024)
    assert tensors["final_layer.audio_out.bias"].ne == (32,)
    end = max(data + t.offset + 4 * int(np.prod(t.ne)) for t in tensors.values())
    assert end <= len(buf)
    try:
        import gguf
    except ImportError:
        return
    r = gguf.GGUFReader(os.path.join(TINY, "dit_globals.bin"))
    for t in r.tensors:
        mine = tensors[t.name]
        a = np.frombuffer(buf, np.float32, int(np.prod(mine.ne)), data + mine.offset)
        np.testing.assert_array_equal(a, np.asarray(t.data, dtype=np.float32).reshape(-1))


def test_rope_tables_match_reference_seq_build(reference):
    from fasth3inc_b200.dit import rope_tables
    pos = np.fromfile(os.path.join(TINY, "pos.bin"), np.float64).reshape(-1, 3)
    pair, c, s = reference.seq_build(6, 4, 8, pos)
    assert list(pair) == [1] * 6 + [2] * 4 + [0] * 8
    c2, s2 = rope_tables(pos)
    np.testing.assert_array_equal(c2, c)
    np.testing.assert_array_equal(s2, s)
    pos = np.random.default_rng(0).uniform(0, 200, (300, 3))
    _, c, s = reference.seq_build(0, 0, 300, pos)
    c2, s2 = rope_tables(pos)
    assert np.abs(c2 - c).max() <= 1.2e-7 and np.abs(s2 - s).max() <= 1.2e-7


def _open_code(fn: str, path: str) -> int:
    import ctypes
    from fasth3inc_b200._lib import load
    h = ctypes.c_void_p()
    if fn == "pack":
        return load().fh3cuda_pack_open(path.encode(), ctypes.byref(h))
    return load().fh3cuda_adaln_open(path.encode(), 0, ctypes.byref(h))


@pytest.mark.skipif(HAS_GPU, reason="checks the file-only path that stops at the missing device")
@pytest.mark.parametrize("fn,name", [("pack", "dit_trunk.bin"), ("adaln", "adaln_table.bin")])
def test_readers_error_codes(tmp_path, fn, name):
    good = open(os.path.join(TINY, name), "rb").read()
    assert _open_code(fn, str(tmp_path / "missing.bin")) == -2                  # FH3_E_IO
    cases = {
        "short": good[:100],                                                      # FH3_E_TRUNCATED
        "magic": b"XXXX" + good[4:],                                              # FH3_E_BAD_MAGIC
        "version": good[:4] + struct.pack("<I", 2) + good[8:],                    # FH3_E_BAD_VERSION
        "cut": good[:len(good) // 2],                                             # tables / layers past the end
    }
    want = {"short": -3, "magic": -4, "version": -5, "cut": -3}
    for k, b in cases.items():
        p = tmp_path / f"{k}.bin"
        p.write_bytes(b)
        assert _open_code(fn, str(p)) == want[k], k
    if fn == "pack":
        p = tmp_path / "align.bin"
        p.write_bytes(good[:12] + struct.pack("<I", 512) + good[16:])
        assert _open_code(fn, str(p)) == -8                                      # FH3_E_INVALID
    assert _open_code(fn, os.path.join(TINY, name)) == -22                      # the file checks out: no device


def _tiny_globals():
    from fasth3inc_b200.dit import read_gguf
    _, tensors, buf, data = read_gguf(os.path.join(TINY, "dit_globals.bin"))
    out = {}
    for name, t in tensors.items():
        a = np.frombuffer(buf, np.float32, int(np.prod(t.ne)), data + t.offset)
        out[name] = a.reshape(tuple(reversed(t.ne))) if len(t.ne) > 1 else a
    return out


def _tiny_inputs():
    from fasth3inc_b200.dit import rope_tables
    f = lambda n, shape: np.fromfile(os.path.join(TINY, n), np.float32).reshape(shape)
    cos, sin = rope_tables(np.fromfile(os.path.join(TINY, "pos.bin"), np.float64))
    return f("text_rows.bin", (6, 256)), f("x_video.bin", (8, 96)), f("x_audio.bin", (4, 32)), cos, sin


TINY_CFG = dict(hidden=256, heads=2, head_dim=128, ffn=512, eps=1e-5, qk_eps=1e-5, final_eps=1e-5, vsa_tile=64,
                vsa_sparsity=0.8)
TINY_SEQ = (18, 6, 4, 8, 1, 1, 8)


@pytest.mark.parametrize("attn,suffix", [(0, ""), (1, "_vsa")])
@pytest.mark.parametrize("step", [0, 7])
def test_oracle_dit_composition_matches_reference_tiny(oracle, attn, suffix, step):
    """The CPU composition used to check the Q4_K DiT forward (tests/q4k_pack.py) reproduces the
    reference's own tiny-model outputs (computed by torch, tests/unit/test_dit_tiny.c:155-156:
    relative L2 <= 1e-4) from the F32 trunk, so it is pinned before it judges the GPU."""
    from conftest import rel_l2
    from q4k_pack import oracle_forward, read_adaln, read_pack
    layers = read_pack(os.path.join(TINY, "dit_trunk.bin"))
    text_rows, xv, xa, cos, sin = _tiny_inputs()
    vv, va = oracle_forward(oracle, layers, _tiny_globals(), read_adaln(os.path.join(TINY, "adaln_table.bin")),
                            text_rows, xv, xa, cos, sin, step, dict(TINY_CFG, attn=attn), TINY_SEQ)
    ref_v = np.fromfile(os.path.join(TINY, f"video_v{suffix}_step{step}.bin"), np.float32).reshape(vv.shape)
    ref_a = np.fromfile(os.path.join(TINY, f"audio_v{suffix}_step{step}.bin"), np.float32).reshape(va.shape)
    assert rel_l2(vv, ref_v) <= 1e-4 and rel_l2(va, ref_a) <= 1e-4


def test_q4k_pack_rewrite_passes_the_readers_file_checks(tmp_path, oracle):
    """The synthetic Q4_K pack keeps the FH3P layout: every projection becomes Q4_K rows of the
    same shape, norms stay F32, and (without a device) fh3cuda_pack_open accepts the file up to
    the device allocation."""
    from q4k_pack import read_pack, write_q4k_pack
    dst = str(tmp_path / "q4k_trunk.bin")
    src_layers = read_pack(os.path.join(TINY, "dit_trunk.bin"))
    write_q4k_pack(os.path.join(TINY, "dit_trunk.bin"), dst, oracle)
    got = read_pack(dst)
    assert len(got) == len(src_layers) == 3
    for a, b in zip(got, src_layers):
        for name in ("qkv", "out", "fc1", "fc2"):
            assert a[name]["type"] == 12 and (a[name]["in_"], a[name]["out"]) == (b[name]["in_"], b[name]["out"])
            assert len(a[name]["raw"]) == a[name]["out"] * oracle.row_bytes(12, a[name]["in_"])
            deq = oracle.dequant(12, a[name]["raw"], a[name]["out"], a[name]["in_"])
            w = b[name]["raw"].view(np.float32).reshape(deq.shape)
            assert np.abs(deq - w).max() <= 0.1 * np.abs(w).max()       # a Q4_K rounding of the same weights
        for name in ("norm1", "norm2", "q_norm", "k_norm"):
            assert a[name]["type"] == 0 and np.array_equal(a[name]["raw"], b[name]["raw"])
    if not HAS_GPU:
        assert _open_code("pack", dst) == -22                  # the file checks out: no device
