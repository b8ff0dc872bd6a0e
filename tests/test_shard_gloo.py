"""The N-shard bookkeeping of the multi-GPU path, run as 2 and 3 gloo ranks on CPU: each rank
takes its rows of B / scales / zero points with the plan of csrc/sharded.cu, computes its
columns with the oracle, all-gathers, and the unsharded result equals the unsharded oracle. The
same runs once more with each rank reading only its byte ranges of an ONNX external data file,
narrowed as tq4_sharded_create_from narrows them."""

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


def _rank_file(rank, world, port, n, m, path, offsets, q):
    """One rank reading only its rows of B, scales and zero points from the data file."""
    from oracle import matmul_nbits as o
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = workloads.Config("shard-gloo-file", 96, n, m, zp="packed", scale_type="f16")
        p = workloads.make(cfg)
        first, count = sharded.shard_rows(n, world, rank)
        share = sharded.shard_share(n, world)
        part = np.zeros((m, share), np.float32)
        if count:
            got = []
            with open(path, "rb") as f:
                for key, dtype in (("B", np.uint8), ("scales", np.float16), ("zp", np.uint8)):
                    off, length = sharded.shard_range(offsets[key], p[key].nbytes, n, world, rank)
                    f.seek(off)
                    got.append(np.frombuffer(f.read(length), dtype=dtype))
            b = got[0].reshape(count, cfg.blocks, -1)
            y, _ = o.matmul_nbits(dict(p["attrs"], N=count), p["A"], b, got[1], got[2])
            part[:, :count] = y
        out = [torch.zeros(m, share) for _ in range(world)]
        dist.all_gather(out, torch.from_numpy(part))
        y_all = sharded.unshard(torch.stack(out), m, n, world).numpy()
        y_ref, _ = o.matmul_nbits(p["attrs"], p["A"], p["B"], p["scales"], p["zp"])
        q.put((rank, o.rel_l2(y_all, y_ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,m", [(2, 100, 2), (3, 40, 1)])
def test_gloo_sharded_file_ranges(world, n, m, tmp_path):
    cfg = workloads.Config("shard-gloo-file", 96, n, m, zp="packed", scale_type="f16")
    p = workloads.make(cfg)
    path, offsets, blob = str(tmp_path / "data"), {}, bytearray(b"\0" * 3)
    for key in ("B", "scales", "zp"):
        offsets[key] = len(blob)
        blob += np.ascontiguousarray(p[key]).tobytes()
    (tmp_path / "data").write_bytes(bytes(blob))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_file, args=(r, world, port, n, m, path, offsets, q)) for r in range(world)]
    for proc in procs:
        proc.start()
    results = [q.get(timeout=120) for _ in procs]
    for proc in procs:
        proc.join(timeout=60)
        assert proc.exitcode == 0
    assert all(err < 1e-6 for _, err in results), results
    # the ranks' ranges tile each input exactly
    for key in ("B", "scales", "zp"):
        ranges = [sharded.shard_range(offsets[key], p[key].nbytes, n, world, r) for r in range(world)]
        assert sum(length for _, length in ranges) == p[key].nbytes
        assert ranges[0][0] == offsets[key]
