"""Failure detection without a GPU fault (the reference's counterpart is a watchdog that flags a
call making no progress, test/support/hang_watchdog.exs:1-40, and run_nodes re-raising with the
op and shapes, lib/transmuter.ex:661-679).

- Device side: every wait in the kernels is bounded by a per-device limit (tq4_set_wait_limit).
  A wait on a flag that nothing sets must give up after that limit, report its code in the device
  status word, and leave the context usable for the next call on the same stream.
- Host side: joining a two-rank communicator that the second rank never joins must end with
  TQ4_ERR_TIMEOUT after the caller's deadline, the communicator aborted. It runs in a child
  process, so that whatever NCCL leaves behind ends with that process."""

import ctypes
import json
import os
import subprocess
import sys
import time

import numpy as np
import pytest
import torch

from oracle import matmul_nbits as o
from transmuter_b200 import _lib, workloads
from transmuter_b200.quantized import PackedWeight

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEV = "cuda:0"
PEER_TIMEOUT = 0x106


def device_status():
    code = ctypes.c_int32()
    _lib.check(_lib.load().tq4_device_status(0, ctypes.byref(code)))
    return code.value


def test_peer_wait_runs_out_and_the_stream_stays_usable():
    lib = _lib.load()
    cfg = workloads.Config("failure-after", 1024, 3072, 1)
    p = workloads.make(cfg)
    w = PackedWeight((cfg.k, cfg.n, 4, 32), torch.from_numpy(p["B"]).to(DEV), torch.from_numpy(p["scales"]).to(DEV),
                     dtype=torch.float32, device=DEV)
    a = torch.from_numpy(p["A"]).to(DEV)
    assert device_status() == 0
    _lib.check(lib.tq4_set_wait_limit(0, 2_000_000))  # about a millisecond
    try:
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        t0 = time.perf_counter()
        _lib.check(lib.tq4_selftest_peer_wait(0, stream))
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert device_status() == PEER_TIMEOUT
        assert elapsed < 0.5, elapsed  # the short limit, not the default second
    finally:
        _lib.check(lib.tq4_set_wait_limit(0, 0))
    # the same stream then runs an ordinary call, with the default limit back
    y = w.matmul(a)
    torch.cuda.synchronize()
    ref, _ = o.matmul_nbits(p["attrs"], p["A"], p["B"], p["scales"], None)
    assert o.rel_l2(y.double().cpu().numpy(), ref) < 1e-3
    assert device_status() == 0


def test_wait_limit_is_checked():
    lib = _lib.load()
    assert lib.tq4_set_wait_limit(0, 10) == 1  # below the smallest limit
    assert lib.tq4_set_wait_limit(0, -5) == 1
    assert lib.tq4_set_wait_limit(99, 0) == 1  # no such device
    _lib.check(lib.tq4_set_wait_limit(0, 0))


CHILD = r"""
import ctypes, json, os, sys, time
sys.path.insert(0, sys.argv[1])
from transmuter_b200 import _lib
lib = _lib.load()
buf = ctypes.create_string_buffer(_lib.UNIQUE_ID_BYTES)
_lib.check(lib.tq4_comm_unique_id(buf))
handle = ctypes.c_void_p()
t0 = time.perf_counter()
st = lib.tq4_comm_create(buf.raw, 2, 0, 0, 3000, ctypes.byref(handle))
print(json.dumps({"status": st, "elapsed": time.perf_counter() - t0, "handle": handle.value,
                  "error": _lib.last_error()}), flush=True)
os._exit(0)
"""


def test_communicator_times_out_when_a_rank_never_joins():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-c", CHILD, ROOT], env=env,
                       capture_output=True, text=True, timeout=150)
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    assert lines, r.stdout[-2000:] + r.stderr[-2000:]
    out = json.loads(lines[-1])
    assert out["status"] == 6, out  # TQ4_ERR_TIMEOUT
    assert "timed out" in out["error"]
    assert out["handle"] is None  # no communicator is handed out; it was aborted
    assert 2.5 < out["elapsed"] < 60, out
