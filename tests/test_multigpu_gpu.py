"""Row-sharded trunk step on 2 GPUs over NCCL must equal the single-GPU step bit for bit.

Every projection is row-independent and each output element's K-accumulation order is
fixed by the kernel, so sharding rows across ranks (fasth3inc_b200.trunk.rows_for_rank)
and all-gathering them at the end reproduces the unsharded step exactly.  Skipped when
fewer than 2 GPUs are visible."""
from __future__ import annotations

import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _n_gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_rank(rank, world, port, M, T, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import fasth3inc_b200 as fh3
        from fasth3inc_b200.trunk import Runner, Trunk, Workspace, rows_for_rank
        d, F = 512, 1024
        trunk = Trunk(d=d, F=F, n_blocks=2, seed=11, device=rank).build()
        g = torch.Generator(device=f"cuda:{rank}").manual_seed(5)
        h_full = torch.randn((M, d), device=f"cuda:{rank}", generator=g)
        text = fh3.to_bf16(torch.randn((T, d), device=f"cuda:{rank}", generator=g))
        r0, r1 = rows_for_rank(M, rank, world)
        h = h_full[r0:r1].clone()
        Runner(trunk, Workspace(r1 - r0, T, d=d, F=F, device=rank)).step(h, text)
        shard = (M + world - 1) // world
        send = torch.zeros((shard, d), device=f"cuda:{rank}")
        send[: r1 - r0] = h
        out = torch.empty((shard * world, d), device=f"cuda:{rank}")
        dist.all_gather_into_tensor(out, send)
        gathered = torch.cat([out[r * shard: r * shard + (rows_for_rank(M, r, world)[1] -
                                                          rows_for_rank(M, r, world)[0])]
                              for r in range(world)])
        ok = True
        if rank == 0:
            full = h_full.clone()
            Runner(trunk, Workspace(M, T, d=d, F=F, device=rank)).step(full, text)
            ok = bool(torch.equal(gathered, full))
        torch.cuda.synchronize()
        q.put((rank, ok, fh3.device_status()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("M", [600, 601])
def test_two_gpu_row_sharded_step_is_exact(M):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run_rank, args=(r, 2, port, M, 40, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok and st == 0 for _, ok, st in res)
