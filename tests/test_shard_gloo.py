"""The N-shard bookkeeping of the multi-GPU path, run as 2 and 3 gloo ranks on CPU: each rank
takes its rows of B / scales / zero points with the plan of csrc/sharded.cu, computes its
columns with the oracle, all-gathers, and the unsharded result equals the unsharded oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from transmuter_b200 import sharded, workloads


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_share_plan():
    assert sharded.shard_share(151936, 8) == 18992
    assert sharded.shard_share(4096, 8) == 512
    assert sharded.shard_share(40, 8) == 16
    rows = [sharded.shard_rows(40, 8, r) for r in range(8)]
    assert rows[:3] == [(0, 16), (16, 16), (32, 8)] and all(c == 0 for _, c in rows[3:])
    assert sum(c for _, c in (sharded.shard_rows(151936, 8, r) for r in range(8))) == 151936


def _rank(rank, world, port, n, m, q):
    from oracle import matmul_nbits as o
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = workloads.Config("shard-gloo", 96, n, m, zp="packed")
        p = workloads.make(cfg)
        blocks = cfg.blocks
        first, count = sharded.shard_rows(n, world, rank)
        share = sharded.shard_share(n, world)
        part = np.zeros((m, share), np.float32)
        if count:
            zrow = -(-blocks * cfg.bits // 8)
            zp = p["zp"].reshape(n, zrow)[first:first + count].reshape(-1)
            attrs = dict(p["attrs"], N=count)
            y, _ = o.matmul_nbits(attrs, p["A"], p["B"][first:first + count],
                                  p["scales"].reshape(n, blocks)[first:first + count].reshape(-1), zp)
            part[:, :count] = y
        out = [torch.zeros(m, share) for _ in range(world)]
        dist.all_gather(out, torch.from_numpy(part))
        gathered = torch.stack(out)
        y_all = sharded.unshard(gathered, m, n, world).numpy()
        y_ref, _ = o.matmul_nbits(p["attrs"], p["A"], p["B"], p["scales"], p["zp"])
        q.put((rank, o.rel_l2(y_all, y_ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,m", [(2, 100, 3), (3, 40, 1)])
def test_gloo_sharded_matches_unsharded(world, n, m):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, n, m, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err < 1e-6 for _, err in results), results
