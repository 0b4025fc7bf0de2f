"""Multi-rank host logic of the row-sharded step, on CPU with the gloo backend.

The step shards latent rows across ranks (fasth3inc_b200.trunk.rows_for_rank), runs
the row-independent projections locally and all-gathers padded equal shards at the
end (bench.py).  Here each rank applies a row-wise stand-in for the trunk and the
gathered result must equal the unsharded computation, for even and ragged splits.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, d, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from fasth3inc_b200.trunk import rows_for_rank
        g = torch.Generator().manual_seed(0)
        h_full = torch.randn((total, d), generator=g)
        w = torch.randn((d, d), generator=g)
        r0, r1 = rows_for_rank(total, rank, world)
        local = torch.tanh(h_full[r0:r1] @ w) + h_full[r0:r1]        # row-independent stand-in
        shard = (total + world - 1) // world
        send = torch.zeros((shard, d))
        send[: r1 - r0] = local
        out = torch.empty((shard * world, d))
        dist.all_gather_into_tensor(out, send)
        # reassemble the ragged shards in rank order
        parts = []
        for r in range(world):
            a, b = rows_for_rank(total, r, world)
            parts.append(out[r * shard: r * shard + (b - a)])
        gathered = torch.cat(parts)
        ref = torch.tanh(h_full @ w) + h_full
        q.put((rank, bool(torch.allclose(gathered, ref, atol=1e-5, rtol=1e-5)), gathered.shape[0]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [64, 67])
def test_row_sharded_step_gathers_exactly(total):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, 16, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok and n == total for _, ok, n in res)
