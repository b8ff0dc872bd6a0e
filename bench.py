"""Benchmark of the B200 MatMulNBits hot path (libtq4) on the north-star configs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c3m1] [--impl ours|reference]

A step is one MatMulNBits call (one pass of the hot path over one batch of activations). The
default workload is the lm_head-shaped config C3 at M = 1 (A f32 [1, 1024], K=1024, N=151936,
4-bit, block 32, f32 scales, no zero points; metric HBM GB/s), the first metric the north star
names. Under ``--gpus N`` (torchrun, one rank per GPU) it runs N-sharded: each rank holds 1/N of
the weight rows and Y is assembled on every rank over NVLink (strong scaling). Other workloads:
c1 (decode, M=1, GB/s), c2 (prefill M=512, TFLOP/s), c3m64, c5-<K>x<N>-m<M> (Llama-3-8B shapes;
N-sharded under --gpus N), c4 (the q4 decoder, tok/s; independent replicas under --gpus N).

Timing: W untimed warm-up steps; the K steps are captured in one CUDA graph, which is replayed
back to back (a replay holds K steps, or a multiple of K when K steps take under 2 ms) until the
timed region lasts at least one second, between barriers and synchronizes; CUDA events on the
launching stream, max over ranks; the line gives the replays and the calls timed. Consecutive
steps rotate over R independent copies of (weights, A, Y) whose total exceeds twice the L2, so no
step reads another step's data from L2. `value` has the inputs resident in HBM; `e2e` times the
same calls through the public API with A copied in from pinned host memory and Y read back to
pinned host memory at every step, the copies on two side streams overlapping other steps'
compute (a serving loop's pipeline), ordered by events.

`--impl reference` times the reference's arithmetic on the host cores instead (the CPU oracle's
moved-weight path: weights dequantized once as lib/transmuter.ex:1230-1240 does, then a dense
f32 BLAS product per call, as EXLA's CPU client runs a moved model; `cpu_baseline.in_graph` also
times the per-call unpack + dequantize path of a model that was not moved). CPU figures are the
median of at least 20 calls after 3 warm-up calls (fewer calls, stated in the sample, when one
call exceeds the time budget).
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MatMulNBits q4 HBM GB/s (M=1), TFLOP/s (M>=256); q4 decoder decode tok/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c3m1")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return FALLBACK_PEAKS, "fallback"


def metric_value(cfg, seconds_per_call, full=True):
    if cfg.metric == "TFLOP/s":
        return cfg.flops() / seconds_per_call / 1e12
    return cfg.algorithmic_bytes() / seconds_per_call / 1e9


# ---- clocks ----------------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        self.t0 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        with open(self.file.name) as f:
            rows = [r.strip().split(",") for r in f if r.strip()]
        os.unlink(self.file.name)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except ValueError:
                continue
            for name, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---- reference (CPU) path --------------------------------------------------------------------
_BLAS_LIMITS = None


def use_all_host_threads():
    """The CPU legs use every host core this process may run on, whatever OMP_NUM_THREADS the
    launcher set (torchrun sets 1 per rank)."""
    global _BLAS_LIMITS
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    try:
        from threadpoolctl import threadpool_limits
        _BLAS_LIMITS = threadpool_limits(limits=n, user_api="blas")
    except Exception:
        pass


def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        info = [x for x in threadpool_info() if x.get("user_api") == "blas"]
        return max(x.get("num_threads", 1) for x in info) if info else os.cpu_count()
    except Exception:
        return os.cpu_count()


def cpu_reference(cfg, p, steps, warmup, budget_s):
    """The oracle's moved-weight path on the host cores: W dequantized once (not timed), then a
    dense f32 A @ W^T per call. `warmup` (at least 3) untimed calls, then `steps` (at least 20)
    timed calls, fewer only when the calls would exceed budget_s (at least 3). Returns (value in
    the metric's unit from the MEDIAN call time, calls timed, sample text)."""
    use_all_host_threads()
    from oracle import matmul_nbits as o
    t = cfg.scale_type
    w = o.dequantize_weight(p["B"], p["scales"], p["zp"], cfg.k, cfg.n, cfg.bits, cfg.block_size, t)
    w32 = np.ascontiguousarray(w.astype(np.float32))
    del w
    a32 = np.ascontiguousarray(np.asarray(p["A"], np.float32))
    for _ in range(max(3, warmup)):
        a32 @ w32.T
    want = max(20, steps)
    times = []
    t_end = time.perf_counter() + budget_s
    for _ in range(want):
        t0 = time.perf_counter()
        y = a32 @ w32.T
        times.append(time.perf_counter() - t0)
        if len(times) >= 3 and time.perf_counter() > t_end:
            break
    sec = statistics.median(times)
    del y
    sample = (f"oracle moved-weight path (dequantize once, then numpy/BLAS f32 A@W^T): median of "
              f"{len(times)} calls after {max(3, warmup)} warm-up calls, full {cfg.m}x{cfg.k}x{cfg.n} workload")
    return metric_value(cfg, sec), len(times), sample


def in_graph(cfg, p, budget_s=8.0):
    """The in-graph CPU figure as a cpu_baseline entry (the headline value stays the faster
    moved-weight path)."""
    v, n, sample = cpu_in_graph(cfg, p, budget_s)
    return {"value": v, "unit": cfg.metric, "calls": n, "sample": sample}


def cpu_in_graph(cfg, p, budget_s):
    """The oracle's in-graph path on the host cores: each call unpacks and dequantizes W in A's
    type (quantized.ex:42, packed.ex:9-36), then the f32 BLAS A @ W^T. This is what a model that
    was not moved runs per call. At least one call; further calls while within budget_s (at most
    20). Returns (value in the metric's unit from the median call, calls timed, sample text)."""
    from oracle import matmul_nbits as o
    a32 = np.ascontiguousarray(np.asarray(p["A"], np.float32))
    times = []
    t_end = time.perf_counter() + budget_s
    while not times or (time.perf_counter() < t_end and len(times) < 20):
        t0 = time.perf_counter()
        w = o.dequantize_weight(p["B"], p["scales"], p["zp"], cfg.k, cfg.n, cfg.bits, cfg.block_size, cfg.a_type)
        y = a32 @ np.asarray(w, np.float32).T
        times.append(time.perf_counter() - t0)
        del w, y
    sec = statistics.median(times)
    sample = (f"oracle in-graph path (unpack + dequantize in {cfg.a_type} every call, then numpy/BLAS "
              f"f32 A@W^T): median of {len(times)} calls of the full {cfg.m}x{cfg.k}x{cfg.n} workload")
    return metric_value(cfg, sec), len(times), sample


def workload_config(cfg, world):
    """The `config` of both arms' lines (identical, so the two arms name the same run): the
    workload, how the GPU arm splits it over `world` GPUs and how it keeps steps out of L2."""
    sharded = sharded_workload(cfg, world)
    per_copy = cfg.algorithmic_bytes() / (world if sharded else 1)
    copies = rotation_copies(per_copy)
    if sharded:
        par = (f"N-sharded over {world} GPUs (each rank 1/{world} of the weight rows); Y assembled on every rank over "
               f"NVLink (M = 1: each GPU's kernel stores its columns into every rank's buffer)")
    else:
        par = "single GPU" if world == 1 else f"{world} independent replicas (dp{world})"
    return {"workload": cfg.name, "M": cfg.m, "K": cfg.k, "N": cfg.n, "bits": cfg.bits,
            "block_size": cfg.block_size, "scales": cfg.scale_type, "zero_points": cfg.zp,
            "activations": cfg.a_type, "parallelism": par,
            "l2": f"rotating {copies} copies of weights+A+Y per GPU ({copies * per_copy / 2**20:.0f} MiB > 2x L2)"}


def sharded_workload(cfg, world):
    """C3 and C5 are N-sharded across the GPUs; the others run independent replicas."""
    return world > 1 and cfg.name.startswith(("c3", "c5"))


def rotation_copies(per_copy_bytes):
    return min(64, max(2, int(np.ceil(2 * L2_BYTES / per_copy_bytes))))


# ---- our path --------------------------------------------------------------------------------
def roofline_traffic(workload, sharded_world=1, path=None):
    """DRAM bytes of one launch of the workload's dominant kernel, from the committed ncu capture
    (profiles/traffic.json), and where the figure comes from. Under N-sharding a rank streams 1/N
    of the weight rows, which are all but a few KB of the capture: the one-GPU figure / N."""
    path = path or os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None, None
    with open(path) as f:
        traffic = json.load(f).get(workload)
    if traffic is None:
        return None, None
    if sharded_world > 1:
        return traffic / sharded_world, ("the one-GPU capture scaled by the rank's 1/N share of the "
                                         "weight rows (not captured on N GPUs)")
    return traffic, "ncu capture of one launch on one GPU (profiles/traffic.json)"


def launches_per_call(cfg, m, sharded_world=1):
    """libtq4 kernels per call (NCCL's own kernels are not counted)."""
    groups = -(-(cfg.blocks * cfg.block_size * cfg.bits // 8) // 64)   # packed groups of 64 bytes per row
    if m == 1 and cfg.bits == 4 and groups > 8 and cfg.block_size <= 1024:
        n = 2                                   # the K-sliced 32-row-unit GEMV + the sum of its slices
    elif m <= 8:
        n = 1                                   # the GEMV
    else:
        n = 2 if cfg.a_type == "f32" else 1     # (row-scaled f16 copy of A) + the tcgen05 GEMM
    if sharded_world > 1:
        if m == 1 and cfg.bits == 4 and groups <= 8 and sharded_world <= 8:
            return n + 1                        # the assembly kernel of the push path
        share = (-(-cfg.n // sharded_world) + 15) // 16 * 16
        if m * share * (4 if cfg.a_type == "f32" else 2) >= 4 << 20:
            n += 1                              # the NVLink exchange kernel
        elif not (m == 1 and cfg.n % (16 * sharded_world) == 0):
            n += 1                              # the reordering kernel after NCCL's all-gather
    return n


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.workload == "c4":
        return decoder_bench(args, rank, world, local_rank)
    from transmuter_b200 import workloads
    if args.workload not in workloads.CONFIGS:
        raise SystemExit(f"unknown workload {args.workload}; one of {sorted(workloads.CONFIGS)}")
    cfg = workloads.CONFIGS[args.workload]
    config = workload_config(cfg, world)
    sharded_run = sharded_workload(cfg, world)

    if args.impl == "reference":
        if rank != 0:
            return
        steps = args.steps or 20
        p = workloads.make(cfg)
        value, n_timed, sample = cpu_reference(cfg, p, steps, args.warmup, budget_s=120.0)
        cores = blas_threads()
        line = {"impl": "reference", "metric": METRIC, "value": value, "unit": cfg.metric, "n_gpus": world,
                "steps": steps, "warmup": args.warmup, "ms_per_step": metric_to_ms(cfg, value),
                "higher_is_better": True, "scaling": "strong" if sharded_run else "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (seeded; shapes and distributions of the config)",
                "config": config,
                "cpu_baseline": {"value": value, "unit": cfg.metric, "cores": cores, "kind": "port",
                                 "sample": sample + " (the whole workload on the host cores of rank 0)",
                                 "in_graph": in_graph(cfg, p)},
                "e2e": {"value": value, "unit": cfg.metric, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from transmuter_b200.quantized import PackedWeight
    from transmuter_b200 import sharded as shd
    TT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}

    # weak scaling (independent batches per rank) unless the workload is N-sharded
    p = workloads.make(cfg, seed_name=cfg.name if (world == 1 or sharded_run) else f"{cfg.name}/rank{rank}")

    def to_dev(x, t=None):
        if x is None:
            return None
        tt = torch.from_numpy(np.ascontiguousarray(x))
        return (tt.to(torch.bfloat16) if t == "bf16" else tt).to(dev)

    attrs = (cfg.k, cfg.n, cfg.bits, cfg.block_size)
    zp_t = cfg.scale_type if cfg.zp == "float" else None
    per_copy = cfg.algorithmic_bytes() / (world if sharded_run else 1)
    copies = rotation_copies(per_copy)
    comm = None
    if sharded_run:
        uid = shd.Comm.unique_id() if rank == 0 else bytes(128)
        obj = [uid]
        dist.broadcast_object_list(obj, src=0)
        comm = shd.Comm(obj[0], world, rank, local_rank, timeout_ms=120000)
    weights, acts, outs = [], [], []
    b_d, s_d, z_d = to_dev(p["B"]), to_dev(p["scales"], cfg.scale_type), to_dev(p["zp"], zp_t)
    for i in range(copies):
        if sharded_run:
            weights.append(shd.ShardedWeight(comm, attrs, b_d, s_d, z_d, dtype=TT[cfg.scale_type]))
        else:
            weights.append(PackedWeight(attrs, b_d, s_d, z_d, dtype=TT[cfg.scale_type], device=dev))
        acts.append(to_dev(p["A"], cfg.a_type))
        outs.append(torch.empty((cfg.m, cfg.n), dtype=TT[cfg.a_type], device=dev))
    del b_d, s_d, z_d
    stream = torch.cuda.current_stream(dev)

    def step(i):
        j = i % copies
        weights[j].matmul(acts[j], out=outs[j])

    def barrier():
        if world > 1:
            dist.barrier()

    def agree(x, op):
        """The same value on every rank (every rank takes the same steps)."""
        if world > 1:
            t = torch.tensor([x], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=op)
            x = t.item()
        return x

    for i in range(max(3, args.warmup)):  # warm-up steps
        step(i)
    torch.cuda.synchronize()
    # per-step time estimate: sizes the default K and the replay count
    t0 = time.perf_counter()
    for i in range(20):
        step(i)
    torch.cuda.synchronize()
    est = agree((time.perf_counter() - t0) / 20, dist.ReduceOp.MAX)
    steps = args.steps or int(min(20000, max(50, 0.05 / max(est, 1e-7))))
    # One replay holds the K steps, or the smallest multiple of K that takes 2 ms, so the graph
    # launch between replays stays a small share of the region.
    per_replay = steps * max(1, int(np.ceil(0.002 / max(steps * est, 1e-9))))

    # The timed steps are one CUDA graph (the calls are launch-bound at small sizes); the graph's
    # stream is warmed first so no workspace is allocated during capture.
    gstream = torch.cuda.Stream(dev)
    with torch.cuda.stream(gstream):
        for i in range(max(3, args.warmup, copies)):  # every copy: its workspaces exist before capture
            step(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gstream):
        for i in range(per_replay):
            step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # one untimed replay measures the replay time; then enough replays for >= 1 s
    barrier()
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    # (sized for 1.2 s: the measured replay is a cold one, the timed replays run warm)
    replays = int(agree(max(1, int(np.ceil(1200.0 / max(e0.elapsed_time(e1), 1e-3)))),
                        dist.ReduceOp.MAX))

    sampler = ClockSampler(local_rank)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(replays):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms_total = agree(e0.elapsed_time(e1), dist.ReduceOp.MAX)
    del graph
    timed_calls = replays * per_replay
    ms = ms_total / timed_calls  # per step
    sec_per_call = ms / 1e3
    units = world if not sharded_run else 1
    value = metric_value(cfg, sec_per_call) * units

    # e2e through the public API: every step copies its A in from pinned host memory and its Y out
    # to pinned host memory, pipelined as a serving loop runs it: the copies of one step overlap
    # other steps' compute on two side streams (in, out), ordered by events; a rotating device
    # buffer (and host buffer) is reused only once the step that used it is done with it.
    a_host = torch.from_numpy(np.ascontiguousarray(p["A"]))
    a_host = (a_host.to(torch.bfloat16) if cfg.a_type == "bf16" else a_host).pin_memory()
    y_hosts = [torch.empty((cfg.m, cfg.n), dtype=TT[cfg.a_type]).pin_memory() for _ in range(copies)]
    s_in, s_out, s_cap = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def pipelined(n, comp):
        copied_in, computed, copied_out = [None] * n, [None] * n, [None] * n
        for i in range(n):
            j = i % copies
            with torch.cuda.stream(s_in):
                if i >= copies:
                    s_in.wait_event(computed[i - copies])  # acts[j] no longer read
                acts[j].copy_(a_host, non_blocking=True)
                copied_in[i] = torch.cuda.Event()
                copied_in[i].record(s_in)
            comp.wait_event(copied_in[i])
            if i >= copies:
                comp.wait_event(copied_out[i - copies])  # outs[j] already read back
            step(i)
            computed[i] = torch.cuda.Event()
            computed[i].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[i])
                y_hosts[j].copy_(outs[j], non_blocking=True)
                copied_out[i] = torch.cuda.Event()
                copied_out[i].record(s_out)

    # The pipeline of n_cap steps is one CUDA graph (the host would otherwise bound a ~20 us step):
    # the side streams fork from the capture stream and join it at the end.
    n_cap = copies * max(1, -(-48 // copies))
    with torch.cuda.stream(s_cap):  # workspaces of the capture stream exist before the capture
        s_in.wait_stream(s_cap)
        s_out.wait_stream(s_cap)
        pipelined(copies, s_cap)
        s_cap.wait_stream(s_in)
        s_cap.wait_stream(s_out)
    torch.cuda.synchronize()
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e, stream=s_cap):
        s_in.wait_stream(s_cap)
        s_out.wait_stream(s_cap)
        pipelined(n_cap, s_cap)
        s_cap.wait_stream(s_in)
        s_cap.wait_stream(s_out)
    g_e2e.replay()
    torch.cuda.synchronize()
    reps = int(agree(max(2, int(np.ceil(0.5 / max(est * n_cap, 1e-6)))), dist.ReduceOp.MAX))
    e2e_steps = reps * n_cap
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(reps):
        g_e2e.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    del g_e2e
    ms_e2e = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = t.item()
    e2e_value = metric_value(cfg, ms_e2e / 1e3 / e2e_steps) * units

    # roofline of the dominant kernel (the MatMulNBits kernel is the whole step; with N-sharding
    # each GPU's kernel does 1/world of the work within the step)
    pk, pk_kind = peaks()
    launches = launches_per_call(cfg, cfg.m, world if sharded_run else 1)
    if cfg.metric == "TFLOP/s":
        achieved = cfg.flops() / (world if sharded_run else 1) / sec_per_call / 1e12
        peak = pk["bf16_tflops"]
        bound, unit = "tensor", "TFLOP/s"
    else:
        achieved = cfg.algorithmic_bytes() / (world if sharded_run else 1) / sec_per_call / 1e9
        peak = pk["hbm_gbs"]
        bound, unit = "hbm", "GB/s"
    traffic, traffic_source = roofline_traffic(args.workload, world if sharded_run else 1)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": cfg.metric, "n_gpus": world, "steps": steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "replays": replays, "steps_per_replay": per_replay, "timed_steps": timed_calls,
                "timed_region_ms": ms_total,
                "scaling": "strong" if sharded_run else "weak", "vs_baseline": None,
                "dtype": cfg.a_type, "data": "synthetic (seeded; shapes and distributions of the config)",
                "config": config,
                "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                             "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_source,
                             "peak_source": f"{pk_kind} ({'burst' if bound == 'tensor' else 'copy'})",
                             "scope": ("one GPU's share of the whole step (its 1/N of the weight through the "
                                       "MatMulNBits kernel, plus the assembly of Y)") if sharded_run else
                                      "the MatMulNBits kernel (the whole step)"},
                "e2e": {"value": e2e_value, "unit": cfg.metric,
                        "h2d_bytes_per_step": int(a_host.numel() * a_host.element_size()),
                        "d2h_bytes_per_step": int(y_hosts[0].numel() * y_hosts[0].element_size()),
                        "steps": e2e_steps,
                        "copies": "every step: A in from pinned host memory, Y out to pinned host memory, on "
                                  "two side streams overlapping other steps' compute (one CUDA graph of "
                                  f"{n_cap} steps per replay)"},
                "gpu_launches": timed_calls * launches, "clocks": clocks}
        if world == 1 and not args.no_cpu_baseline:
            v, n_timed, sample = cpu_reference(cfg, p, 20, 3, budget_s=20.0)
            line["cpu_baseline"] = {"value": v, "unit": cfg.metric, "cores": blas_threads(), "kind": "port",
                                    "sample": sample, "in_graph": in_graph(cfg, p)}
        print(json.dumps(line), flush=True)

    for w in weights:
        w.close()
    if comm is not None:
        comm.close()
    if world > 1:
        dist.destroy_process_group()


# ---- C4: the q4 decoder ----------------------------------------------------------------------
DECODE_PROMPT = 128


def decoder_bytes_per_token(cfg, pos):
    """Algorithmic HBM bytes of one decode step at position `pos`: every MatMulNBits weight once
    (packed nibbles + f32 scales; the embedding row gather is one lm_head row) plus the KV cache
    read up to pos and written at pos (f32)."""
    qkv_n = (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim
    per_layer = cfg.hidden * qkv_n + cfg.heads * cfg.head_dim * cfg.hidden + cfg.hidden * 2 * cfg.inter \
        + cfg.inter * cfg.hidden
    weights = cfg.layers * per_layer + cfg.vocab * cfg.hidden
    packed = weights // 2 + weights // cfg.block_size * 4
    kv = cfg.layers * 2 * cfg.kv_heads * cfg.head_dim * 4 * (pos + 1)
    return packed + kv


def decoder_cpu(cfg, seed, steps, budget_s):
    """Moved-weight CPU path (oracle decoder in float32: dense weights, BLAS matrix-vector products)
    for a bounded number of decode steps at positions 127.. with the cache rows before them
    filled with seeded values (the attention work of a 128-token prefill, without running it)."""
    use_all_host_threads()
    from oracle.decoder import OracleDecoder
    from transmuter_b200.decoder import random_weights, rope_tables
    weights = random_weights(cfg, seed)
    cos, sin = rope_tables(cfg)
    ref = OracleDecoder(cfg, weights, cos, sin, dtype=np.float32)
    del weights
    r = np.random.default_rng(seed)
    fill = (cfg.layers, cfg.kv_heads, DECODE_PROMPT - 1, cfg.head_dim)
    ref.k_cache[:, :, :DECODE_PROMPT - 1] = r.standard_normal(fill, dtype=np.float32)
    ref.v_cache[:, :, :DECODE_PROMPT - 1] = r.standard_normal(fill, dtype=np.float32)
    tok = int(r.integers(0, cfg.vocab))
    ref.step(tok, DECODE_PROMPT - 1)  # warm-up (overwrites its own position)
    times = []
    t_end = time.perf_counter() + budget_s
    for i in range(steps):
        t0 = time.perf_counter()
        tok = int(np.argmax(ref.step(tok, DECODE_PROMPT - 1 + i)))
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end:
            break
    sample = (f"oracle decoder in f32 with dense dequantized weights (numpy/BLAS), {len(times)} greedy decode "
              f"steps from position {DECODE_PROMPT - 1} (cache rows before it seeded, not prefilled)")
    return len(times) / sum(times), len(times), sample


def decoder_bench(args, rank, world, local_rank):
    """Decode tok/s of the Qwen3-0.6B-shaped q4 decoder: a 128-token prompt (forced steps, timed
    separately as prefill), then K greedy decode steps, each one CUDA graph replay of a whole
    token (28 layers, lm_head, argmax) with the position and token in device memory. N > 1 runs
    independent replicas (the decoder does not shard)."""
    import zlib
    from transmuter_b200.decoder import QWEN3_0_6B, Q4Decoder, random_weights, split_siblings
    cfg = QWEN3_0_6B
    seed = zlib.crc32(b"c4")
    config = {"workload": "c4 Qwen3-0.6B-shaped q4 decoder, batch 1, f32 KV cache",
              "layers": cfg.layers, "hidden": cfg.hidden, "inter": cfg.inter, "heads": cfg.heads,
              "kv_heads": cfg.kv_heads, "head_dim": cfg.head_dim, "vocab": cfg.vocab, "block_size": cfg.block_size,
              "scales": "f32", "prompt_tokens": DECODE_PROMPT}
    steps = args.steps or 128
    if steps > cfg.max_len - DECODE_PROMPT:
        raise SystemExit(f"--steps at most {cfg.max_len - DECODE_PROMPT} for c4 (cache of {cfg.max_len})")
    # the same config for both arms (the driver compares them)
    config["parallelism"] = "single GPU" if world == 1 else f"{world} independent replicas"
    if args.impl == "reference":
        if rank != 0:
            return
        value, n_timed, sample = decoder_cpu(cfg, seed, steps, budget_s=120.0)
        line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
                "steps": steps, "warmup": args.warmup, "ms_per_step": 1e3 / value, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (random-init weights of the architecture, seeded prompt)", "config": config,
                "cpu_baseline": {"value": value, "unit": "tok/s", "cores": blas_threads(), "kind": "port",
                                 "sample": sample + f" ({n_timed} of {steps} steps timed)"},
                "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    # q, k, v and gate, up as separate inputs (as an ONNX export stores them), merged at load
    dec = Q4Decoder(cfg, device=dev, weights=split_siblings(random_weights(cfg, seed), cfg))
    prompt = np.random.default_rng(seed + rank).integers(0, cfg.vocab, DECODE_PROMPT)
    dec.reset(prompt)
    dec.capture()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(ms):
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms

    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    for _ in range(max(3, args.warmup)):  # warm-up: whole sequences
        dec.reset(prompt)
        dec.run(DECODE_PROMPT - 1 + steps)
    torch.cuda.synchronize()
    dec.reset(prompt)
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    dec.run(DECODE_PROMPT - 1)  # prefill: forced prompt tokens
    e1.record(stream)
    dec.run(steps)              # timed decode steps
    e2.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms_prefill = max_over_ranks(e0.elapsed_time(e1))
    ms = max_over_ranks(e1.elapsed_time(e2))
    tokens = dec.log[DECODE_PROMPT:DECODE_PROMPT + steps].cpu().numpy()
    value = steps / (ms / 1e3) * world

    # e2e through the public API: generate() copies the prompt in and the tokens out
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t0.record(stream)
    out = dec.generate(prompt, steps)
    t1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = max_over_ranks(t0.elapsed_time(t1))
    assert np.array_equal(out, tokens), "generate() and the timed decode disagree"

    pk, pk_kind = peaks()
    step_bytes = np.mean([decoder_bytes_per_token(cfg, DECODE_PROMPT - 1 + i) for i in range(steps)])
    achieved = step_bytes / (ms / 1e3 / steps) / 1e9
    launches = cfg.layers * Q4Decoder.LAUNCHES_PER_LAYER + Q4Decoder.LAUNCHES_PER_STEP_EXTRA
    if rank == 0:
        config["l2"] = "inputs larger than L2 (about 372 MB of weights read per token, L2 126 MB)"
        config["prefill"] = {"tok_per_s": (DECODE_PROMPT - 1) / (ms_prefill / 1e3) * world,
                             "note": "prompt run as forced decode steps (M=1), one graph replay per token"}
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
                "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (random-init weights of the architecture, seeded prompt)", "config": config,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": achieved / pk["hbm_gbs"], "traffic": None,
                             "scope": "whole decode step (all launches of one token); bytes = weights + KV",
                             "peak_source": f"{pk_kind} (copy)"},
                "e2e": {"value": steps / (ms_e2e / 1e3) * world, "unit": "tok/s",
                        "h2d_bytes_per_step": int(DECODE_PROMPT * 8 // steps),
                        "d2h_bytes_per_step": 8,
                        "note": "generate(): prompt in, prefill, decode, tokens out; tok/s counts decode tokens"},
                "gpu_launches": steps * launches, "clocks": clocks}
        if world == 1 and not args.no_cpu_baseline:
            del dec
            torch.cuda.empty_cache()
            v, n_timed, sample = decoder_cpu(cfg, seed, steps, budget_s=20.0)
            line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": blas_threads(), "kind": "port",
                                    "sample": sample}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def metric_to_ms(cfg, value):
    if cfg.metric == "TFLOP/s":
        return cfg.flops() / (value * 1e12) * 1e3
    return cfg.algorithmic_bytes() / (value * 1e9) * 1e3


if __name__ == "__main__":
    main()
