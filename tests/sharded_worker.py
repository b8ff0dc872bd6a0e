"""One rank of the N-sharded MatMulNBits GPU test (launched by tests/test_gpu_sharded.py through
torch.distributed.run, one process per GPU).

Every rank builds the same seeded weights, takes its rows through tq4_sharded_create (and, for one
weight, through tq4_sharded_create_from reading an external data file), runs
tq4_sharded_matmul twice in a row on different inputs (its GEMV / GEMM, then the assembly of Y:
NCCL's all-gather for small outputs, the NVLink peer exchange for slices of 4 MB and more) and
compares the full Y with the unsharded handle on its own GPU. The columns come from
the same kernels over the same rows, so they agree to within the split-K summation order
(rel-L2 1e-6 for f32 outputs; 1e-4 for f16 outputs, where that order can move a value by one
f16 ulp); the unsharded result is itself pinned to the oracle by the parity tests.
Exit status 0 when every case agrees on every rank.
"""

import json
import os
import sys
import tempfile
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle import matmul_nbits as o  # noqa: E402
from transmuter_b200 import sharded, workloads  # noqa: E402
from transmuter_b200.deferred import DeferredTensor, TensorProto  # noqa: E402
from transmuter_b200.quantized import PackedWeight  # noqa: E402

CASES = [  # (K, N, M, zero points, A type, scale type)
    (1024, 151936, 1, "none", "f32", "f32"),
    (1024, 151936, 3, "none", "f32", "f32"),
    (4096, 14336, 1, "packed", "f16", "f16"),
    (1024, 4000, 64, "packed", "f16", "f16"),
    (4096, 1024, 256, "packed", "f16", "f16"),
    # slices of 4 MB and more per rank: the NVLink peer exchange instead of NCCL's all-gather
    (4096, 14336, 512, "packed", "f16", "f16"),
    (1024, 151936, 16, "none", "f32", "f32"),
    # M = 1 with at most 8 packed groups per row: each rank's GEMV pushes its columns into every
    # rank's assembly buffer (ragged N; a last rank with few rows; f16 outputs)
    (1000, 4099, 1, "packed", "f16", "f16"),
    (1024, 40, 1, "none", "f32", "f32"),
]
TT = {"f32": torch.float32, "f16": torch.float16}


def external_case(comm, rank, dev):
    """The same weight as ONNX external data (tq4_sharded_create_from): each rank reads only its
    rows of the file, and its Y must equal the one built from memory, bit for bit."""
    k, n, bs = 4096, 14336, 128
    cfg = workloads.Config("shard-gpu-external", k, n, 4, block_size=bs, zp="packed", a_type="f16", scale_type="f16")
    p = workloads.make(cfg)
    where = [tempfile.mkdtemp(prefix="tq4-shard-") if rank == 0 else None]
    dist.broadcast_object_list(where, src=0)
    d = where[0]
    arrays = [("B", p["B"], 2), ("scales", p["scales"], 10), ("zero_points", p["zp"], 2)]
    if rank == 0:
        with open(os.path.join(d, "data"), "wb") as f:
            f.write(b"\0" * 7)
            for _, arr, _ in arrays:
                f.write(np.ascontiguousarray(arr).tobytes())
    dist.barrier()
    deferred, off = [], 7
    for i, (name, arr, ty) in enumerate(arrays):
        entries = [("location", "data"), ("offset", str(off))] + ([("length", str(arr.nbytes))] if i < 2 else [])
        deferred.append(DeferredTensor.new(TensorProto(name, list(arr.shape), ty, "EXTERNAL", entries), d))
        off += arr.nbytes
    mem = [torch.from_numpy(np.ascontiguousarray(arr)).to(dev) for _, arr, _ in arrays]
    a = torch.from_numpy(np.ascontiguousarray(p["A"])).to(dev)
    sw_f = sharded.ShardedWeight(comm, (k, n, 4, bs), *deferred, dtype=torch.float16)
    sw_m = sharded.ShardedWeight(comm, (k, n, 4, bs), *mem, dtype=torch.float16)
    y_f, y_m = sw_f.matmul(a), sw_m.matmul(a)
    torch.cuda.synchronize()
    exact = torch.equal(y_f, y_m) and (sw_f.first, sw_f.count) == (sw_m.first, sw_m.count)
    sw_f.close()
    sw_m.close()
    dist.barrier()
    if rank == 0:
        os.remove(os.path.join(d, "data"))
        os.rmdir(d)
    return ("shard-gpu-external", 0.0 if exact else 1.0, 0.5)


def push_graph_case(comm, rank, dev):
    """The M = 1 push path with a bias, captured in a CUDA graph of three calls (alternating
    inputs) and replayed twice: the epoch that picks the assembly half lives in device memory, so
    replays keep advancing it. Every call must equal the eager unsharded one."""
    k, n = 1024, 151936
    cfg = workloads.Config("shard-gpu-push-graph", k, n, 1, bias=True)
    p = workloads.make(cfg)
    b, s = torch.from_numpy(p["B"]).to(dev), torch.from_numpy(p["scales"]).to(dev)
    bias = torch.from_numpy(p["bias"]).to(dev)
    a = torch.from_numpy(np.ascontiguousarray(p["A"])).to(dev)
    ins = [a, torch.flip(a, dims=[1]).contiguous(), -a]
    sw = sharded.ShardedWeight(comm, (k, n, 4, 32), b, s, None, dtype=torch.float32)
    pw = PackedWeight((k, n, 4, 32), b, s, None, dtype=torch.float32, device=dev)
    refs = [pw.matmul(x, bias) for x in ins]
    outs = [torch.empty(1, n, device=dev) for _ in ins]
    gs = torch.cuda.Stream(dev)
    with torch.cuda.stream(gs):
        for x, y in zip(ins, outs):  # warm-up outside the capture (maps peer memory once)
            sw.matmul(x, bias, out=y)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gs):
        for x, y in zip(ins, outs):
            sw.matmul(x, bias, out=y)
    worst = 0.0
    for _ in range(2):
        for y in outs:
            y.zero_()
        graph.replay()
        torch.cuda.synchronize()
        for y, ref in zip(outs, refs):
            worst = max(worst, o.rel_l2(y.double().cpu().numpy(), ref.double().cpu().numpy()))
    del graph
    sw.close()
    pw.close()
    return ("shard-gpu-push-graph", worst, 1e-6)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    uid = [sharded.Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = sharded.Comm(uid[0], world, rank, rank, timeout_ms=60000)
    worst = []
    for k, n, m, zp, at, st in CASES:
        bs = 32 if k == 1024 else 128
        cfg = workloads.Config(f"shard-gpu-{k}x{n}-m{m}", k, n, m, block_size=bs, zp=zp, a_type=at, scale_type=st)
        p = workloads.make(cfg)
        b = torch.from_numpy(p["B"]).to(dev)
        s = torch.from_numpy(p["scales"]).to(dev)
        z = torch.from_numpy(p["zp"]).to(dev) if p["zp"] is not None else None
        a = torch.from_numpy(np.ascontiguousarray(p["A"])).to(dev)
        sw = sharded.ShardedWeight(comm, (k, n, 4, bs), b, s, z, dtype=TT[st])
        pw = PackedWeight((k, n, 4, bs), b, s, z, dtype=TT[st], device=dev)
        a2 = torch.flip(a, dims=[1]).contiguous()  # a second call in a row, on new inputs
        y_sh, y_sh2 = sw.matmul(a), sw.matmul(a2)
        y_ref, y_ref2 = pw.matmul(a), pw.matmul(a2)
        torch.cuda.synchronize()
        err = max(o.rel_l2(y_sh.double().cpu().numpy(), y_ref.double().cpu().numpy()),
                  o.rel_l2(y_sh2.double().cpu().numpy(), y_ref2.double().cpu().numpy()))
        worst.append((cfg.name, err, 1e-6 if at == "f32" else 1e-4))
        sw.close()
        pw.close()
    worst.append(external_case(comm, rank, dev))
    worst.append(push_graph_case(comm, rank, dev))
    comm.close()
    ok = all(e < tol for _, e, tol in worst)
    flags = torch.tensor([int(ok)])
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(json.dumps({"world": world, "ok": bool(flags.item()), "cases": worst}), flush=True)
    dist.destroy_process_group()
    sys.exit(0 if flags.item() else 1)


if __name__ == "__main__":
    main()
