"""GPU tests of the N-sharded MatMulNBits path (tq4_comm_* / tq4_sharded_*): a one-rank
communicator in this process, and two ranks (one process per GPU, NCCL all-gather over NVLink)
through tests/sharded_worker.py when the box has two GPUs. The sharded Y must equal the
unsharded handle's Y on the same GPU to within the split-K summation order."""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import matmul_nbits as o
from transmuter_b200 import sharded, workloads
from transmuter_b200.deferred import DeferredTensor, TensorProto
from transmuter_b200.quantized import PackedWeight

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("m", [1, 4, 40])
def test_one_rank_sharded_equals_unsharded(m):
    dev = torch.device("cuda:0")
    cfg = workloads.Config(f"shard-one-{m}", 1024, 3000, m, zp="packed", a_type="f16", scale_type="f16")
    p = workloads.make(cfg)
    b, s = torch.from_numpy(p["B"]).to(dev), torch.from_numpy(p["scales"]).to(dev)
    z = torch.from_numpy(p["zp"]).to(dev)
    a = torch.from_numpy(p["A"]).to(dev)
    comm = sharded.Comm(sharded.Comm.unique_id(), 1, 0, 0, timeout_ms=30000)
    sw = sharded.ShardedWeight(comm, (1024, 3000, 4, 32), b, s, z, dtype=torch.float16)
    pw = PackedWeight((1024, 3000, 4, 32), b, s, z, dtype=torch.float16, device=dev)
    assert (sw.first, sw.count) == (0, 3000)
    y_sh, y_ref = sw.matmul(a), pw.matmul(a)
    torch.cuda.synchronize()
    assert torch.equal(y_sh, y_ref)  # one rank: the same kernel over the same rows
    ref, _ = o.matmul_nbits(p["attrs"], p["A"], p["B"], p["scales"], p["zp"])
    assert o.rel_l2(y_sh.double().cpu().numpy(), ref) < 5e-3
    sw.close()
    pw.close()
    comm.close()


def test_one_rank_sharded_from_external_data(tmp_path):
    """tq4_sharded_create_from: the rank's rows read from an external data file give the Y of
    the same rows given in memory."""
    dev = torch.device("cuda:0")
    cfg = workloads.Config("shard-one-external", 1024, 3000, 3, zp="packed", a_type="f16", scale_type="f16")
    p = workloads.make(cfg)
    arrays = [("B", p["B"], 2), ("scales", p["scales"], 10), ("zero_points", p["zp"], 2)]
    blob, deferred = bytearray(b"\1" * 5), []
    for name, arr, ty in arrays:
        entries = [("location", "data"), ("offset", str(len(blob))), ("length", str(arr.nbytes))]
        deferred.append(DeferredTensor.new(TensorProto(name, list(arr.shape), ty, "EXTERNAL", entries), str(tmp_path)))
        blob += np.ascontiguousarray(arr).tobytes()
    (tmp_path / "data").write_bytes(bytes(blob))
    a = torch.from_numpy(p["A"]).to(dev)
    comm = sharded.Comm(sharded.Comm.unique_id(), 1, 0, 0, timeout_ms=30000)
    sw_f = sharded.ShardedWeight(comm, (1024, 3000, 4, 32), *deferred, dtype=torch.float16)
    sw_m = sharded.ShardedWeight(comm, (1024, 3000, 4, 32), *[torch.from_numpy(x).to(dev) for _, x, _ in arrays],
                                 dtype=torch.float16)
    assert torch.equal(sw_f.matmul(a), sw_m.matmul(a))
    sw_f.close()
    sw_m.close()
    comm.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_sharded_equals_unsharded():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29517",
           os.path.join(ROOT, "tests", "sharded_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert '"ok": true' in r.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 3, reason="needs more than two GPUs")
def test_all_ranks_sharded_equals_unsharded():
    """The same cases on every GPU of the box (up to 8 ranks): ragged shares, a last rank with few
    or no rows, both assembly paths and the M = 1 push path with 2 < P <= 8 destinations."""
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29518",
           os.path.join(ROOT, "tests", "sharded_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=500)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert f'"world": {n}, "ok": true' in r.stdout
