"""One rank of the N-sharded MatMulNBits GPU test (launched by tests/test_gpu_sharded.py through
torch.distributed.run, one process per GPU).

Every rank builds the same seeded weights, takes its rows through tq4_sharded_create, runs
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
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle import matmul_nbits as o  # noqa: E402
from transmuter_b200 import sharded, workloads  # noqa: E402
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
]
TT = {"f32": torch.float32, "f16": torch.float16}


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
