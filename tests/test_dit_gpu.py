"""The tiny end-to-end DiT (the reference's tests/fixtures/tiny_h3) on the GPU.

The trunk (FH3P) and the AdaLN table (FH3A) are read once into HBM (fh3cuda_pack_open /
fh3cuda_adaln_open) and must hold the file's bytes; the globals come from the GGUF file.
fh3cuda_dit_prepare_text_dev and fh3cuda_dit_forward_dev must meet the reference's own bar
against torch's outputs, relative L2 <= 1e-4 (tests/unit/test_dit_tiny.c:155-156), with fp32
attention, for dense and video sparse attention at steps 0 and 7.  With bf16 tensor-core
attention the bar is 2e-2.
"""
from __future__ import annotations

import ctypes
import os
import struct

import numpy as np
import pytest

from conftest import GOLDEN, rel_l2

pytestmark = pytest.mark.gpu
TINY = os.path.join(GOLDEN, "tiny_h3")
TOL = 1e-4
SEQ = (18, 6, 4, 8, 1, 1, 8)     # text 6 | audio 4 | video 8 (grid fallback 1 x 1 x 8)


def _f32(name, shape=None):
    a = np.fromfile(os.path.join(TINY, name), np.float32)
    return a.reshape(shape) if shape else a


def _dev_floats(addr: int, n: int):
    """Copy n fp32 values at a device address (a type-F32 'dequant' is a copy)."""
    import torch
    from fasth3inc_b200._lib import check, load
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    check(load().fh3cuda_dequant_dev(0, ctypes.c_void_p(addr), ctypes.c_void_p(out.data_ptr()), 1, n, None))
    return out.cpu().numpy()


def _cfg(attn=0, bf16=0):
    from fasth3inc_b200._lib import Fh3CudaDitCfg
    # tests/unit/test_dit_tiny.c:77-101
    return Fh3CudaDitCfg(attn=attn, vsa_tile=64, vsa_sparsity=0.8, hidden_size=256, num_heads=2, head_dim=128,
                         num_layers=3, num_refiner_layers=2, ffn_dim=512, norm_eps=1e-5, qk_norm_eps=1e-5,
                         final_norm_eps=1e-5, attn_bf16=bf16)


@pytest.fixture(scope="module")
def model(fh3):
    import torch
    from fasth3inc_b200.dit import Adaln, DitGlobals, Pack, rope_tables
    pack = Pack(os.path.join(TINY, "dit_trunk.bin"))
    adaln = Adaln(os.path.join(TINY, "adaln_table.bin"))
    glob = DitGlobals(os.path.join(TINY, "dit_globals.bin"), 2)
    cos, sin = rope_tables(np.fromfile(os.path.join(TINY, "pos.bin"), np.float64))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    inputs = dict(cos=dev(cos), sin=dev(sin), x_video=dev(_f32("x_video.bin", (8, 96))),
                  x_audio=dev(_f32("x_audio.bin", (4, 32))), text_emb=dev(_f32("text_emb.bin", (6, 64))))
    yield pack, adaln, glob, inputs
    pack.close()
    adaln.close()


def test_pack_resident_bytes_equal_the_file(model):
    pack = model[0]
    buf = open(os.path.join(TINY, "dit_trunk.bin"), "rb").read()
    nl = struct.unpack_from("<I", buf, 8)[0]
    index_off, index_bytes = struct.unpack_from("<QQ", buf, 16)
    assert pack.num_layers == nl == 3 and pack.device_bytes > 0
    names = ("qkv", "gate_compress", "out", "fc1", "fc2", "norm1", "norm2", "q_norm", "k_norm")
    for L in range(nl):
        d = index_off + L * (index_bytes // nl)
        file_off = struct.unpack_from("<Q", buf, d)[0]
        v = pack.layer(L)
        for t, nm in enumerate(names):
            td = d + 24 + 168 * t
            typ = struct.unpack_from("<I", buf, td + 64)[0]
            off, size, in_, out = struct.unpack_from("<QQqq", buf, td + 104)
            w = getattr(v, nm)
            assert (w.type, w.in_, w.out) == (typ, in_, out), (L, nm)
            assert typ == 0                                    # the tiny trunk is F32
            n = size // 4
            np.testing.assert_array_equal(_dev_floats(w.data, n),
                                          np.frombuffer(buf, np.float32, n, file_off + off))


def test_adaln_rows_equal_the_file(model):
    adaln = model[1]
    buf = open(os.path.join(TINY, "adaln_table.bin"), "rb").read()
    n_steps, n_blocks, pairs, hidden = struct.unpack_from("<IIII", buf, 8)
    trunk_off, _, final_off, _ = struct.unpack_from("<QQQQ", buf, 32)
    assert (adaln.n_steps, adaln.n_blocks, adaln.pairs, adaln.hidden) == (n_steps, n_blocks, pairs, hidden)
    for step, blk, pair, ch in ((0, 0, 0, 0), (7, 2, 2, 5), (3, 1, 1, 3)):
        idx = (((step * n_blocks + blk) * pairs + pair) * 6 + ch) * hidden
        np.testing.assert_array_equal(_dev_floats(adaln.row(step, blk, pair, ch), hidden),
                                      np.frombuffer(buf, np.float32, hidden, trunk_off + 4 * idx))
    idx = ((5 * pairs + 1) * 2 + 1) * hidden
    np.testing.assert_array_equal(_dev_floats(adaln.row(5, -1, 1, 1), hidden),
                                  np.frombuffer(buf, np.float32, hidden, final_off + 4 * idx))
    assert adaln.row(8, 0, 0, 0) is None and adaln.row(0, 0, 3, 0) is None and adaln.row(0, 0, 0, 6) is None


def test_prepare_text_matches_torch(model):
    from fasth3inc_b200.dit import Dit
    _, _, glob, x = model
    rows = Dit(_cfg(), glob).prepare_text(x["text_emb"]).cpu().numpy()
    assert rel_l2(rows, _f32("text_rows.bin", (6, 256))) <= TOL


@pytest.mark.parametrize("attn,step", [(0, 0), (0, 7), (1, 0), (1, 7)])
def test_forward_matches_torch(model, attn, step):
    from fasth3inc_b200.dit import Dit
    pack, adaln, glob, x = model
    dit = Dit(_cfg(attn), glob)
    rows = dit.prepare_text(x["text_emb"])
    vv, va = dit.forward(pack, adaln, SEQ, x["cos"], x["sin"], step, x["x_video"], x["x_audio"], rows)
    tag = "_vsa" if attn else ""
    assert rel_l2(vv.cpu().numpy(), _f32(f"video_v{tag}_step{step}.bin", (8, 96))) <= TOL
    assert rel_l2(va.cpu().numpy(), _f32(f"audio_v{tag}_step{step}.bin", (4, 32))) <= TOL


@pytest.mark.parametrize("attn", [0, 1])
def test_forward_bf16_attention(model, attn):
    from fasth3inc_b200.dit import Dit
    pack, adaln, glob, x = model
    dit = Dit(_cfg(attn, bf16=1), glob)
    rows = dit.prepare_text(x["text_emb"])
    vv, va = dit.forward(pack, adaln, SEQ, x["cos"], x["sin"], 0, x["x_video"], x["x_audio"], rows)
    tag = "_vsa" if attn else ""
    assert rel_l2(vv.cpu().numpy(), _f32(f"video_v{tag}_step0.bin", (8, 96))) <= 2e-2
    assert rel_l2(va.cpu().numpy(), _f32(f"audio_v{tag}_step0.bin", (4, 32))) <= 2e-2


def test_forward_rejects_step_outside_the_table(model):
    from fasth3inc_b200 import Fh3CudaError
    from fasth3inc_b200.dit import Dit
    pack, adaln, glob, x = model
    dit = Dit(_cfg(), glob)
    rows = dit.prepare_text(x["text_emb"])
    with pytest.raises(Fh3CudaError) as e:
        dit.forward(pack, adaln, SEQ, x["cos"], x["sin"], 8, x["x_video"], x["x_audio"], rows)
    assert e.value.code == -8
