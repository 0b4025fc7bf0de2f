"""The DiT forward on a Q4_K trunk: the reference's tiny model (tests/golden/tiny_h3) with its
projections quantised to Q4_K and repacked in the FH3P layout by tests/q4k_pack.py.

With bf16 tensor-core attention every trunk block then runs on bf16 operands with the GEMMs'
fused prologue and epilogues (rmsnorm+modulate -> QKV -> q/k norm+rope in bf16 -> attention ->
O with the gated residual in its epilogue -> rmsnorm+modulate -> fc1 with SwiGLU -> fc2 with
the gated residual): the launches of the bench's trunk.  The result is checked against the
oracle's fp32 composition of fh3_dit_forward on the same Q4_K weights (that composition
reproduces the reference's own outputs from the F32 trunk within 1e-4,
tests/test_dit_host.py).  Bar: relative L2 <= 2e-2, the bf16 tensor-core bar of the tiny
model's tests; the fp32-attention chain of the same trunk is held to it too."""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import GOLDEN, rel_l2

pytestmark = pytest.mark.gpu
TINY = os.path.join(GOLDEN, "tiny_h3")
SEQ = (18, 6, 4, 8, 1, 1, 8)
TOL = 2e-2


@pytest.fixture(scope="module")
def q4k_model(fh3, oracle, tmp_path_factory):
    import torch
    from fasth3inc_b200.dit import Adaln, DitGlobals, Pack, rope_tables
    from q4k_pack import read_adaln, write_q4k_pack
    from test_dit_host import _tiny_globals, _tiny_inputs
    path = str(tmp_path_factory.mktemp("q4k") / "q4k_trunk.bin")
    layers = write_q4k_pack(os.path.join(TINY, "dit_trunk.bin"), path, oracle)
    pack = Pack(path)
    adaln_path = os.path.join(TINY, "adaln_table.bin")
    text_rows, xv, xa, cos, sin = _tiny_inputs()
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    yield dict(pack=pack, adaln=Adaln(adaln_path), glob=DitGlobals(os.path.join(TINY, "dit_globals.bin"), 2),
               layers=layers, host_glob=_tiny_globals(), host_adaln=read_adaln(adaln_path),
               host=(text_rows, xv, xa, cos, sin), dev=[dev(a) for a in (text_rows, xv, xa, cos, sin)])


@pytest.mark.parametrize("attn_bf16", [1, 0])
@pytest.mark.parametrize("attn", [0, 1])
@pytest.mark.parametrize("step", [0, 7])
def test_q4k_trunk_forward_vs_oracle(fh3, oracle, q4k_model, attn_bf16, attn, step):
    from fasth3inc_b200._lib import Fh3CudaDitCfg
    from fasth3inc_b200.dit import Dit
    from q4k_pack import oracle_forward
    from test_dit_host import TINY_CFG
    m = q4k_model
    cfg = Fh3CudaDitCfg(attn=attn, vsa_tile=64, vsa_sparsity=0.8, hidden_size=256, num_heads=2, head_dim=128,
                        num_layers=3, num_refiner_layers=2, ffn_dim=512, norm_eps=1e-5, qk_norm_eps=1e-5,
                        final_norm_eps=1e-5, attn_bf16=attn_bf16)
    text_rows, xv, xa, cos, sin = m["dev"]
    vv, va = Dit(cfg, m["glob"]).forward(m["pack"], m["adaln"], SEQ, cos, sin, step, xv, xa, text_rows)
    assert fh3.device_status() == 0
    ht, hxv, hxa, hcos, hsin = m["host"]
    rv, ra = oracle_forward(oracle, m["layers"], m["host_glob"], m["host_adaln"], ht, hxv, hxa, hcos, hsin, step,
                            dict(TINY_CFG, attn=attn), SEQ)
    assert rel_l2(vv.cpu().numpy(), rv) <= TOL
    assert rel_l2(va.cpu().numpy(), ra) <= TOL
