"""bench.py's bookkeeping on CPU: the libtq4 launches it claims per call for each workload's path
(the line's `gpu_launches`), and the config both arms print."""

import bench
from transmuter_b200 import workloads

C = workloads.CONFIGS


def test_launches_per_call():
    assert bench.launches_per_call(C["c3m1"], 1) == 1                 # 32-row-unit GEMV
    assert bench.launches_per_call(C["c1"], 1) == 1
    assert bench.launches_per_call(C["c5-4096x14336-m1"], 1) == 2     # K-sliced GEMV + slice sum
    assert bench.launches_per_call(C["c5-14336x4096-m1"], 1) == 2
    assert bench.launches_per_call(C["c2"], C["c2"].m) == 1           # tcgen05 GEMM, f16 A
    assert bench.launches_per_call(C["c3m64"], 64) == 2               # row-scaled f16 copy of A + GEMM
    assert bench.launches_per_call(C["c5-4096x14336-m16"], 16) == 1   # GEMM on a 32-row tile
    assert bench.launches_per_call(C["c5-4096x4096-m4096"], 4096) == 1
    # N-sharded M = 1 lm_head: the GEMV plus the push path's assembly kernel
    for n in (2, 4, 8):
        assert bench.launches_per_call(C["c3m1"], 1, sharded_world=n) == 2


def test_both_arms_print_one_config():
    for name in ("c3m1", "c2", "c5-4096x14336-m1"):
        for world in (1, 2, 8):
            assert bench.workload_config(C[name], world) == bench.workload_config(C[name], world)
            assert "parallelism" in bench.workload_config(C[name], world)


def test_roofline_traffic(tmp_path):
    path = tmp_path / "traffic.json"
    path.write_text('{"c3m1": 100000000}')
    assert bench.roofline_traffic("c3m1", 1, str(path))[0] == 100000000
    t, src = bench.roofline_traffic("c3m1", 4, str(path))
    assert t == 25000000 and "1/N" in src
    assert bench.roofline_traffic("c2", 1, str(path)) == (None, None)
    assert bench.roofline_traffic("c3m1", 1, str(tmp_path / "absent.json")) == (None, None)
    # the committed captures: one per benchmarked GEMV / GEMM workload named in them
    t, _ = bench.roofline_traffic("c3m1")
    assert t is not None and t > workloads.CONFIGS["c3m1"].algorithmic_bytes()
