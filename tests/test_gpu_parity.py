"""GPU parity of the tq4 kernels against the CPU oracle, through the C ABI (ctypes).

Bars (north star): dequantized weights bit-exact; outputs within rel-L2 1e-3 for f32
activations and 5e-3 for f16/bf16 activations; the reference fixtures within the reference's
own tolerance (ops_test.exs:582-598)."""

import numpy as np
import pytest
import torch

from oracle import matmul_nbits as o
from tests.golden_cases import gather_cases, matmul_nbits_cases
from transmuter_b200 import quantized, workloads
from transmuter_b200.quantized import ArgumentError, Node, PackedWeight

pytestmark = pytest.mark.gpu

TOL = {"f32": 1e-3, "f16": 5e-3, "bf16": 5e-3}
TORCH = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
DEV = "cuda:0"


def to_dev(x, t=None):
    if x is None:
        return None
    tt = torch.from_numpy(np.ascontiguousarray(x))
    if t == "bf16":
        tt = tt.to(torch.bfloat16)
    return tt.to(DEV)


def as_np32(t):
    return t.float().cpu().numpy()


def device_status():
    import ctypes
    from transmuter_b200 import _lib
    code = ctypes.c_int32()
    _lib.check(_lib.load().tq4_device_status(0, ctypes.byref(code)))
    return code.value


def weight_for(cfg, p, dtype):
    return PackedWeight((cfg.k, cfg.n, cfg.bits, cfg.block_size), to_dev(p["B"]),
                        to_dev(p["scales"], cfg.scale_type), to_dev(p["zp"], cfg.scale_type if cfg.zp == "float" else None),
                        dtype=TORCH[dtype], device=DEV)


# ---- the reference's fixtures through the operator entry point ------------------------------

@pytest.mark.parametrize("case", matmul_nbits_cases(), ids=lambda c: c["name"])
def test_reference_fixture(case):
    ins = (case["inputs"] + [None] * 6)[:6]
    a, b, scales, zp, g_idx, bias = ins
    node = Node("MatMulNBits", case["attrs"], case["input_names"])
    inputs = [to_dev(a), to_dev(b), to_dev(scales), to_dev(zp), None, to_dev(bias)]
    (y,) = quantized.apply(node, inputs)
    y = as_np32(y)
    diff, tol = o.within_reference_tolerance(y, case["Y"])
    assert diff <= tol, (diff, tol)
    assert o.rel_l2(y, case["Y"]) < 1e-3


@pytest.mark.parametrize("case", matmul_nbits_cases(), ids=lambda c: c["name"])
def test_reference_fixture_moved(case):
    """The moved weight (Transmuter.move/2) gives the in-graph dequantize, bit for bit."""
    a, b, scales, zp = (case["inputs"] + [None] * 4)[:4]
    k, n, bits, bs = o.nbits_sizes(case["attrs"])
    node = Node("MatMulNBits", case["attrs"], case["input_names"])
    w = quantized.move_weight(node, to_dev(b), to_dev(scales), to_dev(zp), device=DEV)
    got = as_np32(w.dequantize())
    want = o.dequantize_weight(b, scales, zp, k, n, bits, bs, "f32")
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("case", gather_cases(), ids=lambda c: c["name"])
def test_gather_block_quantized_fixture(case):
    data, indices, scales, zp = case["inputs"][:4]
    node = Node("GatherBlockQuantized", case["attrs"], case["input_names"])
    (y,) = quantized.apply(node, [to_dev(data), to_dev(indices), to_dev(scales), to_dev(zp)])
    np.testing.assert_array_equal(as_np32(y), case["Y"])


# ---- bit-exact dequantize over the layout and type space -------------------------------------

DEQ = [
    # bits, bs, K, N, zp, scale type, T
    (4, 32, 1024, 200, "none", "f32", "f32"),
    (4, 16, 72, 40, "packed", "f32", "f32"),
    (4, 32, 72, 17, "none", "f16", "f16"),
    (4, 128, 4096, 64, "packed", "f16", "f16"),
    (4, 256, 768, 33, "float", "f32", "f32"),
    (4, 64, 320, 48, "float", "f16", "f16"),
    (4, 32, 256, 24, "packed", "bf16", "bf16"),
    (4, 32, 256, 24, "packed", "f16", "f32"),
    (2, 16, 64, 8, "packed", "f32", "f32"),
    (2, 32, 544, 31, "none", "f16", "f16"),
    (2, 64, 512, 16, "float", "bf16", "bf16"),
    (8, 32, 64, 8, "packed", "f32", "f32"),
    (8, 16, 200, 21, "none", "f16", "f16"),
    (8, 128, 384, 64, "float", "f32", "bf16"),
]


@pytest.mark.parametrize("bits,bs,k,n,zp,st,t", DEQ)
def test_dequantize_bit_exact(bits, bs, k, n, zp, st, t):
    cfg = workloads.Config(f"deq-{bits}-{bs}-{k}-{n}-{zp}-{st}-{t}", k, n, 1, bits=bits, block_size=bs,
                           scale_type=st, zp=zp, scale_range=(0.001, 2.0))
    p = workloads.make(cfg)
    w = weight_for(cfg, p, t)
    got = as_np32(w.dequantize())
    want = o.dequantize_weight(p["B"], p["scales"], p["zp"], k, n, bits, bs, t).astype(np.float32)
    assert got.shape == want.shape
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


# ---- GEMV (M <= 16) and the large-M path ------------------------------------------------------

GEMV = [
    # K, N, M, bits, bs, zp, scale type, A type, T, bias
    (1024, 3072, 1, 4, 32, "none", "f32", "f32", "f32", False),
    (1024, 3072, 1, 4, 32, "packed", "f16", "f16", "f16", False),
    (1024, 3072, 16, 4, 32, "packed", "f16", "f16", "f16", True),
    (4096, 1024, 1, 4, 128, "packed", "f16", "f16", "f16", False),
    (4096, 1024, 7, 4, 128, "packed", "f16", "f16", "f16", False),
    (14336, 512, 3, 4, 128, "packed", "f16", "f16", "f16", False),
    (72, 16, 6, 4, 32, "none", "f32", "f32", "f32", True),
    (512, 40, 6, 4, 256, "packed", "f32", "f32", "f32", False),
    (1000, 333, 9, 4, 16, "float", "f32", "f32", "f32", True),
    (2048, 500, 5, 4, 64, "packed", "bf16", "bf16", "bf16", False),
    (2048, 500, 12, 4, 64, "none", "f32", "bf16", "f32", False),
    (640, 100, 4, 2, 16, "packed", "f32", "f32", "f32", False),
    (1024, 128, 16, 2, 128, "none", "f16", "f16", "f16", False),
    (640, 100, 4, 8, 32, "packed", "f32", "f32", "f32", False),
    (1024, 96, 11, 8, 16, "float", "f16", "bf16", "f16", True),
    (256, 8, 1, 8, 256, "packed", "bf16", "bf16", "bf16", False),
]


def run_case(k, n, m, bits, bs, zp, st, at, t, bias, scale_range=(0.005, 0.02)):
    cfg = workloads.Config(f"mm-{k}-{n}-{m}-{bits}-{bs}-{zp}-{st}-{at}-{t}-{bias}", k, n, m, bits=bits,
                           block_size=bs, scale_type=st, zp=zp, a_type=at, bias=bias, scale_range=scale_range)
    p = workloads.make(cfg)
    w = weight_for(cfg, p, t)
    a = to_dev(p["A"], at)
    bias_t = to_dev(p["bias"], at) if bias else None
    y = w.matmul(a, bias_t)
    wd = o.dequantize_weight(p["B"], p["scales"], p["zp"], k, n, bits, bs, t)
    want = np.asarray(p["A"], np.float64) @ wd.astype(np.float64).T
    if bias:
        want = want + np.asarray(p["bias"], np.float64)
    return as_np32(y), want, cfg


@pytest.mark.parametrize("k,n,m,bits,bs,zp,st,at,t,bias", GEMV)
def test_gemv_parity(k, n, m, bits, bs, zp, st, at, t, bias):
    got, want, _ = run_case(k, n, m, bits, bs, zp, st, at, t, bias)
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    assert o.rel_l2(got, want) < TOL[at], o.rel_l2(got, want)


@pytest.mark.parametrize("at,bs,bits,zp", [("f32", 128, 4, "none"), ("f32", 32, 4, "packed"), ("f16", 128, 4, "packed"),
                                           ("bf16", 128, 4, "none"), ("f32", 64, 2, "none"), ("f32", 64, 8, "packed")])
@pytest.mark.parametrize("kind", ["positive", "huge", "tiny", "mixed_rows"])
def test_gemv_activation_extremes(at, bs, bits, zp, kind):
    """All-positive activations (the magic-number offset does not cancel), huge and tiny
    magnitudes (the per-segment power-of-two activation scale), and rows of very different size."""
    k, n, m = 4096, 256, 5
    cfg = workloads.Config(f"ext-{at}-{bs}-{bits}-{zp}", k, n, m, bits=bits, block_size=bs, zp=zp,
                           scale_type="f32" if at == "f32" else at, a_type=at)
    p = workloads.make(cfg)
    r = np.random.default_rng(7)
    a = r.random((m, k), dtype=np.float32) * 3.0  # positive
    if kind == "huge":
        a = (r.standard_normal((m, k)) * (1e3 if at == "f16" else 1e30)).astype(np.float32)
    elif kind == "tiny":
        a = (r.standard_normal((m, k)) * (1e-3 if at == "f16" else 1e-30)).astype(np.float32)
    elif kind == "mixed_rows":
        a = r.standard_normal((m, k)).astype(np.float32) * np.array([[1e-3], [1.0], [50.0], [1e-2], [7.0]], np.float32)
    a = o.as_type(a, at) if at != "f32" else a
    w = weight_for(cfg, p, cfg.scale_type)
    y = as_np32(w.matmul(to_dev(np.asarray(a, np.float32) if at == "bf16" else a, at)))
    wd = o.dequantize_weight(p["B"], p["scales"], p["zp"], k, n, bits, bs, cfg.scale_type)
    want = np.asarray(a, np.float64) @ wd.astype(np.float64).T
    for row in range(m):  # each row on its own scale
        assert o.rel_l2(y[row], want[row]) < TOL[at], (row, o.rel_l2(y[row], want[row]))


LARGE_M = [
    (1024, 3072, 17, 4, 32, "packed", "f16", "f16", "f16", False),
    (1024, 256, 64, 4, 32, "none", "f32", "f32", "f32", True),
    (2048, 384, 200, 4, 128, "packed", "f16", "f16", "f16", True),
    (1024, 512, 130, 4, 64, "packed", "bf16", "bf16", "bf16", False),
    (512, 320, 33, 8, 32, "float", "f16", "f16", "f16", False),
    # K split over a cluster of 8 CTAs (few weight-row tiles): f16 with zero points, and f32 A /
    # f32 weights (row scale and weight exponent applied after the cross-CTA sum) with bias
    (4096, 1024, 256, 4, 128, "packed", "f16", "f16", "f16", False),
    (4096, 640, 100, 4, 32, "none", "f32", "f32", "f32", True),
    # blocks that span several 128-k stages (one scale and zero point per stage, read once)
    (2048, 256, 96, 4, 256, "packed", "f16", "f16", "f16", False),
    (2048, 200, 64, 4, 1024, "none", "bf16", "bf16", "bf16", True),
    (3000, 300, 140, 4, 512, "float", "f16", "f16", "f16", True),
]


@pytest.mark.parametrize("k,n,m,bits,bs,zp,st,at,t,bias", LARGE_M)
def test_large_m_parity(k, n, m, bits, bs, zp, st, at, t, bias):
    got, want, _ = run_case(k, n, m, bits, bs, zp, st, at, t, bias)
    assert o.rel_l2(got, want) < TOL[at], o.rel_l2(got, want)


# 2- and 8-bit weights on the tensor-core GEMM (quantized.ex:226-240 takes bits 2, 4 and 8 on one
# path): a stage of 128 k is two packed groups of 8-bit weights or half a group of 2-bit weights.
# K not a multiple of 128 (the last 8-bit stage's second group lies past the row), f32 weights
# (row exponent), bf16 with 8 bits (exact q through f32), narrow tiles (two CTAs per SM) and K
# split over a cluster.
LOW_HIGH_BITS = [
    (1024, 384, 130, 8, 32, "packed", "f16", "f16", "f16", True),
    (320, 256, 64, 8, 32, "none", "f16", "f16", "f16", False),
    (1024, 300, 200, 8, 64, "float", "bf16", "bf16", "bf16", True),
    (512, 256, 129, 8, 128, "packed", "bf16", "bf16", "bf16", False),
    (1024, 256, 48, 8, 32, "none", "f32", "f32", "f32", True),
    (4096, 512, 256, 8, 128, "packed", "f16", "f16", "f16", False),
    (1024, 384, 130, 2, 32, "packed", "f16", "f16", "f16", True),
    (640, 256, 64, 2, 16, "none", "bf16", "bf16", "bf16", False),
    (1024, 300, 200, 2, 64, "float", "f16", "f16", "f16", False),
    (512, 256, 40, 2, 32, "packed", "f32", "f32", "f32", True),
    (4096, 512, 256, 2, 128, "packed", "bf16", "bf16", "bf16", True),
    (1024, 128, 12, 2, 32, "packed", "f16", "f16", "f16", False),
    (1024, 128, 16, 8, 32, "packed", "f16", "bf16", "f16", False),
]


@pytest.mark.parametrize("k,n,m,bits,bs,zp,st,at,t,bias", LOW_HIGH_BITS)
def test_two_and_eight_bit_gemm_parity(k, n, m, bits, bs, zp, st, at, t, bias):
    got, want, _ = run_case(k, n, m, bits, bs, zp, st, at, t, bias)
    assert np.isfinite(got).all()
    assert o.rel_l2(got, want) < TOL[at], o.rel_l2(got, want)


@pytest.mark.parametrize("bits", [2, 8])
def test_two_and_eight_bit_prefill_runs_on_the_tensor_core_gemm(bits):
    """A prefill-sized call with 2- or 8-bit weights is one gemm_kernel launch, not GEMV slices."""
    cfg = workloads.Config(f"route-{bits}", 1024, 512, 256, bits=bits, block_size=32, scale_type="f16",
                           zp="packed", a_type="f16")
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f16")
    a = to_dev(p["A"], "f16")
    w.matmul(a)
    torch.cuda.synchronize()
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        w.matmul(a)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if "kernel" in e.name]
    assert any("gemm_kernel" in n for n in names), names
    assert not any("gemv" in n for n in names), names


# f32 activations at M > 16 take the tensor cores as row-scaled f16 (and f32 weights as
# row-scaled f16); the rel-L2 1e-3 bar of f32 activations still holds, for ordinary, wide and
# tiny scales (the latter would sit in f16's subnormal range without the row exponent).
F32_PREFILL = [
    (1024, 384, 48, 32, "none", (0.005, 0.02)),
    (1000, 333, 40, 16, "float", (0.005, 0.02)),
    (2048, 500, 100, 64, "packed", (0.001, 2.0)),
    (72, 16, 20, 32, "none", (0.005, 0.02)),
    (1024, 256, 64, 32, "packed", (1e-6, 1e-5)),
    (4096, 640, 300, 128, "packed", (0.002, 0.01)),
    (1024, 384, 48, 128, "none", (0.005, 0.02)),   # f16 block scales of f32 weights, one per stage
    (2048, 256, 64, 256, "none", (1e-6, 1e-5)),
]


@pytest.mark.parametrize("k,n,m,bs,zp,scale_range", F32_PREFILL)
def test_f32_prefill_parity(k, n, m, bs, zp, scale_range):
    got, want, _ = run_case(k, n, m, 4, bs, zp, "f32", "f32", "f32", True, scale_range=scale_range)
    assert o.rel_l2(got, want) < TOL["f32"], o.rel_l2(got, want)


def test_c1_full_size():
    cfg = workloads.CONFIGS["c1"]
    got, want, _ = run_case(cfg.k, cfg.n, cfg.m, 4, 32, "none", "f32", "f32", "f32", False)
    assert o.rel_l2(got, want) < 1e-3


def test_c2_full_size():
    cfg = workloads.CONFIGS["c2"]
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f16")
    y = as_np32(w.matmul(to_dev(p["A"])))
    ref, _ = o.matmul_nbits(p["attrs"], p["A"], p["B"], p["scales"], p["zp"])
    assert o.rel_l2(y, ref) < 5e-3


C5_SHAPES = [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)]


@pytest.mark.parametrize("m", [1, 16, 256, 4096])
@pytest.mark.parametrize("k,n", C5_SHAPES)
def test_c5_full_size(k, n, m):
    """Every Llama-shaped call that bench.py times, at its full size and with its own seeded
    inputs (f16 scales, packed zero points, f16 A), against the oracle's MatMulNBits clause
    (quantized.ex:30-46): M = 1 and 16 take the GEMV / narrow GEMM, M = 256 the K-split cluster
    GEMM on the shapes with few weight-row tiles, M = 4096 the 256-row GEMM tiles. At M = 4096 the
    oracle runs on 48 sampled activation rows (rows are independent)."""
    cfg = workloads.CONFIGS[f"c5-{k}x{n}-m{m}"]
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f16")
    y = w.matmul(to_dev(p["A"]))
    rows = np.arange(m) if m <= 256 else np.sort(np.random.default_rng(5).choice(m, 48, replace=False))
    ref, ref_t = o.matmul_nbits(p["attrs"], p["A"][rows], p["B"], p["scales"], p["zp"])
    assert ref_t == "f16"
    got = as_np32(y[torch.from_numpy(rows).to(DEV)])
    assert np.isfinite(got).all()
    assert o.rel_l2(got, ref) < TOL["f16"], o.rel_l2(got, ref)
    assert device_status() == 0


@pytest.mark.parametrize("name", ["c3m1", "c3m64"])
def test_c3_against_oracle_on_sampled_weight_rows(name):
    """The 151936-column lm_head at M = 1 and 64 (f32 A, f32 scales), each with its own bench seed,
    against the oracle's MatMulNBits clause on 4096 sampled weight rows (output columns are
    independent: the oracle gets those rows of B and of the scales, and N = 4096)."""
    cfg = workloads.CONFIGS[name]
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f32")
    y = as_np32(w.matmul(to_dev(p["A"])))
    cols = np.sort(np.random.default_rng(11).choice(cfg.n, 4096, replace=False))
    attrs = dict(p["attrs"], N=len(cols))
    scales = p["scales"].reshape(cfg.n, cfg.blocks)[cols].reshape(-1)
    ref, _ = o.matmul_nbits(attrs, p["A"], p["B"][cols], scales, None)
    assert o.rel_l2(y[:, cols], ref) < TOL["f32"], o.rel_l2(y[:, cols], ref)
    assert device_status() == 0


def test_c3_lm_head_full_size_property():
    """151936 x 1024 at M = 1 and 64: Y equals A . W^T with W from tq4_dequantize (itself checked
    bit-exact against the oracle on sampled rows), in float64 on the CPU."""
    cfg = workloads.CONFIGS["c3m64"]
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f32")
    wd = w.dequantize()
    rows = np.random.default_rng(1).choice(cfg.n, 64, replace=False)
    sub = o.dequantize_weight(p["B"][rows], p["scales"].reshape(cfg.n, -1)[rows].reshape(-1), None,
                              cfg.k, 64, 4, 32, "f32")
    np.testing.assert_array_equal(as_np32(wd[torch.from_numpy(rows).to(DEV)]).view(np.uint32), sub.view(np.uint32))
    a = to_dev(p["A"])
    for m in (1, 64):
        y = w.matmul(a[:m]).double()
        want = a[:m].double() @ wd.double().T
        err = ((y - want).norm() / want.norm()).item()
        assert err < 1e-3, (m, err)


def test_m_zero_is_a_noop_and_errors_are_status():
    cfg = workloads.Config("err", 64, 8, 1)
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f32")
    y = w.matmul(torch.zeros(0, 64, device=DEV))
    assert y.shape == (0, 8)
    with pytest.raises(ArgumentError):
        w.matmul(torch.zeros(1, 63, device=DEV))
    with pytest.raises(ArgumentError):
        w.matmul(torch.zeros(1, 64, dtype=torch.float64, device=DEV))


def test_repeated_calls_are_deterministic():
    """Split-K reductions sum in a fixed order: the same call gives the same bits."""
    cfg = workloads.CONFIGS["c5-4096x1024-m1"]
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f16")
    a = to_dev(p["A"])
    y0 = w.matmul(a)
    for _ in range(3):
        assert torch.equal(w.matmul(a), y0)


def test_concurrent_streams_do_not_share_workspace():
    cfg = workloads.CONFIGS["c5-4096x1024-m16"]
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f16")
    a = to_dev(p["A"])
    ref = w.matmul(a)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    outs = []
    for s in (s1, s2, s1, s2):
        with torch.cuda.stream(s):
            outs.append(w.matmul(a))
    torch.cuda.synchronize()
    for y in outs:
        assert torch.equal(y, ref)


def test_device_status_clean():
    assert device_status() == 0


HANDOUT_M1 = [
    # K, N, bs, zp, scale type, A type, T, bias: N >= 592 row tiles, the row-tile hand-out
    (1024, 76011, 32, "none", "f32", "f32", "f32", False),
    (1024, 76160, 32, "packed", "f16", "f16", "f16", True),
    (2048, 76800, 16, "float", "f32", "f32", "f32", False),
    (512, 77000, 32, "none", "bf16", "bf16", "bf16", False),
    (1000, 76100, 32, "packed", "f32", "bf16", "f32", True),
    (4096, 75800, 32, "none", "f16", "f32", "f16", False),
]


@pytest.mark.parametrize("k,n,bs,zp,st,at,t,bias", HANDOUT_M1)
def test_m1_row_tile_hand_out(k, n, bs, zp, st, at, t, bias):
    """M = 1 with many row tiles per CTA (the lm_head shape) takes whole row tiles by ticket and
    multiplies with B fragments prebuilt during the activation staging: every activation type,
    blocks of 16 and 32, zero points, bias, ragged N and K. Against an fp64 product over the
    bit-exact dequantized weight; back-to-back calls give the same bits (no partial sums)."""
    cfg = workloads.Config(f"tc-{k}-{n}-{bs}-{zp}-{st}-{at}", k, n, 1, bits=4, block_size=bs, scale_type=st,
                           zp=zp, a_type=at, bias=bias)
    p = workloads.make(cfg)
    w = weight_for(cfg, p, t)
    a = to_dev(p["A"], at)
    bias_t = to_dev(p["bias"], at) if bias else None
    ys = [w.matmul(a, bias_t) for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])
    want = a.double() @ w.dequantize().double().T
    if bias:
        want = want + bias_t.double()
    y = ys[0].double()
    assert torch.isfinite(y).all()
    assert ((y - want).norm() / want.norm()).item() < TOL[at]
    assert device_status() == 0


UNITS_M1 = [
    # K, N, bs, zp, scale type, A type, T, bias: M = 1 with at most 8 packed groups per row (K <= 1024),
    # the 32-row-unit kernel: every block size (16 .. 256), zero-point kind and activation type,
    # K not a multiple of 128 or of the block, N not a multiple of 32, fewer units than CTAs
    (1024, 5000, 16, "float", "f32", "f32", "f32", True),
    (1000, 4099, 32, "packed", "f16", "f16", "f16", True),
    (72, 40, 32, "none", "f32", "f32", "f32", True),
    (512, 20000, 64, "packed", "bf16", "bf16", "bf16", False),
    (896, 9000, 128, "none", "f32", "f32", "f32", False),
    (1024, 12345, 256, "packed", "f32", "f32", "f32", True),
    (768, 600, 32, "none", "f16", "f32", "f16", False),
    (1024, 70001, 32, "none", "f32", "bf16", "f32", False),
    (640, 33, 64, "float", "f16", "f16", "f16", True),
    # rows of more than 8 packed groups run K-sliced (each CTA on one slice of 8 groups for the
    # call, the slices' partial rows added in slice order by the last one to finish a unit): 2 to
    # 14 slices, a last slice of one group, blocks up to 1024 spanning several groups
    (1100, 640, 16, "packed", "f16", "f16", "f16", True),
    (2048, 1000, 32, "none", "f32", "f32", "f32", True),
    (3000, 777, 64, "float", "bf16", "bf16", "bf16", False),
    (4096, 3000, 128, "packed", "f16", "f16", "f16", False),
    (4096, 520, 256, "none", "f32", "f32", "f32", True),
    (5120, 300, 1024, "packed", "f32", "bf16", "f32", False),
    (14336, 600, 128, "packed", "f16", "f16", "f16", True),
]


@pytest.mark.parametrize("k,n,bs,zp,st,at,t,bias", UNITS_M1)
def test_m1_units_kernel(k, n, bs, zp, st, at, t, bias):
    """M = 1 over 32-row units (8 consumer warps, warp w on packed group w, B fragments in
    registers, the last warp of a unit adding the groups' partials): against an fp64 product over
    the bit-exact dequantized weight; three calls in a row give the same bits (the unit tickets
    are back at zero after each call), and the device status stays clean."""
    cfg = workloads.Config(f"units-{k}-{n}-{bs}-{zp}-{st}-{at}-{t}", k, n, 1, bits=4, block_size=bs,
                           scale_type=st, zp=zp, a_type=at, bias=bias)
    p = workloads.make(cfg)
    w = weight_for(cfg, p, t)
    a = to_dev(p["A"], at)
    bias_t = to_dev(p["bias"], at) if bias else None
    ys = [w.matmul(a, bias_t) for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])
    wd = o.dequantize_weight(p["B"], p["scales"], p["zp"], k, n, 4, bs, t)
    want = np.asarray(p["A"], np.float64) @ wd.astype(np.float64).T
    if bias:
        want = want + np.asarray(p["bias"], np.float64)
    got = as_np32(ys[0])
    assert np.isfinite(got).all()
    assert o.rel_l2(got, want) < TOL[at], o.rel_l2(got, want)
    assert device_status() == 0


def test_m1_units_interleaved_handles_on_one_stream():
    """Back-to-back calls of different handles on one stream, without synchronising: each handle's
    unit tickets are its own and every call starts from a counter at zero."""
    cfgs = [workloads.Config(f"inter-{i}", 1024, n, 1) for i, n in enumerate((151936, 3072, 40000))]
    ps = [workloads.make(c) for c in cfgs]
    ws = [weight_for(c, p, "f32") for c, p in zip(cfgs, ps)]
    a = [to_dev(p["A"]) for p in ps]
    first = [w.matmul(x) for w, x in zip(ws, a)]
    again = []
    for _ in range(3):
        again.append([w.matmul(x) for w, x in zip(ws, a)])
    torch.cuda.synchronize()
    for rnd in again:
        for y0, y in zip(first, rnd):
            assert torch.equal(y0, y)
    for w, x, y in zip(ws, a, first):
        want = x.double() @ w.dequantize().double().T
        assert ((y.double() - want).norm() / want.norm()).item() < 1e-3
    assert device_status() == 0


def test_lm_head_row_tiles_handed_out_in_arrival_order():
    """The 151936-row lm_head at M = 1 hands whole row tiles to CTAs through an arrival counter
    that the last CTA resets: back-to-back calls on one handle (the next call's prefetch overlaps
    the previous call) must each see a fresh hand-out, and the result has no partial sums, so
    every call gives the same bits whatever CTA took which tile."""
    cfg = workloads.CONFIGS["c3m1"]
    p = workloads.make(cfg)
    w = weight_for(cfg, p, "f32")
    a = to_dev(p["A"])
    a2 = torch.flip(a, dims=[1]).contiguous()
    ys = [w.matmul(x) for x in (a, a2, a, a2, a)]  # no synchronisation between the calls
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[2]) and torch.equal(ys[0], ys[4]) and torch.equal(ys[1], ys[3])
    wd = w.dequantize().double()
    for x, y in ((a, ys[0]), (a2, ys[1])):
        want = x.double() @ wd.T
        assert ((y.double() - want).norm() / want.norm()).item() < 1e-3


MERGE = [
    # K, part N, bs, zp, scale type, T: Qwen3's q/k/v (f32 scales) and gate/up; f16 with packed
    # zero points; float zero points; 2- and 8-bit weights
    (1024, (2048, 1024, 1024), 32, "none", "f32", "f32"),
    (1024, (3072, 3072), 32, "none", "f32", "f32"),
    (4096, (1000, 333, 17), 128, "packed", "f16", "f16"),
    (640, (64, 100), 64, "float", "bf16", "bf16"),
    (512, (40, 24), 32, "packed", "f32", "f32"),
]


@pytest.mark.parametrize("k,parts,bs,zp,st,t", MERGE)
@pytest.mark.parametrize("bits", [4, 2, 8])
def test_merged_siblings(k, parts, bs, zp, st, t, bits):
    """tq4_weight_merge (the packed form of Fusion.matmuls/2, lib/transmuter/fusion.ex:430-540):
    the merged handle's dequantized weight is the row concatenation of the parts', bit for bit,
    and one call gives every part's Y (the Split): the same bits where each row's arithmetic does
    not depend on N (M = 1 over 32-row units), within the summation order otherwise."""
    ws, ps = [], []
    for i, n in enumerate(parts):
        cfg = workloads.Config(f"merge-{k}-{n}-{i}-{bs}-{zp}-{st}-{bits}", k, n, 1, bits=bits, block_size=bs,
                               scale_type=st, zp=zp, a_type=t)
        ps.append(workloads.make(cfg, m=40))
        ws.append(weight_for(cfg, ps[-1], t))
    merged = PackedWeight.merge(ws)
    assert merged.n == sum(parts)
    want = torch.cat([w.dequantize() for w in ws], dim=0)
    got = merged.dequantize()
    assert torch.equal(got.view(torch.int16 if t != "f32" else torch.int32),
                       want.view(torch.int16 if t != "f32" else torch.int32))
    a = to_dev(ps[0]["A"], t)
    for m in (1, 40):
        y = merged.matmul(a[:m])
        ys = torch.cat([w.matmul(a[:m]) for w in ws], dim=1)
        torch.cuda.synchronize()
        if m == 1 and bits == 4 and k <= 1024:  # the 32-row-unit kernel: per-row arithmetic
            assert torch.equal(y, ys), (y - ys).abs().max()
        else:  # split-K plans follow N, so the summation order may differ
            assert ((y.double() - ys.double()).norm() / ys.double().norm()).item() < 1e-3
    for w in ws:  # the parts stay valid after the merge
        w.close()
    y1 = merged.matmul(a[:1])
    torch.cuda.synchronize()
    assert torch.isfinite(y1).all()
    assert device_status() == 0


# ---- signed (s8) data: GatherBlockQuantized tables of int4/int2 exports ----------------------

SIGNED = [
    # bits, block_size, K, rows, zero points ("none", "u8", "s8"), scale type
    (4, 32, 256, 50, "none", "f32"),
    (4, 16, 96, 33, "u8", "f16"),
    (4, 64, 320, 20, "s8", "bf16"),
    (2, 32, 128, 17, "none", "f16"),
    (2, 16, 64, 9, "u8", "f32"),
    (2, 32, 160, 12, "s8", "bf16"),
    (8, 32, 64, 11, "none", "bf16"),
    (8, 16, 48, 7, "u8", "f16"),
    (8, 32, 96, 10, "s8", "f32"),
]


def signed_table(bits, bs, k, rows, zp, st, seed):
    rng = np.random.default_rng(seed)
    data = rng.integers(-128, 128, size=(rows, k * bits // 8), dtype=np.int16).astype(np.int8)
    blocks = -(-k // bs)
    scales = rng.uniform(0.01, 0.5, size=(rows, blocks)).astype(np.float32)
    scales = scales.astype(np.float16) if st == "f16" else scales
    zrow = -(-blocks * bits // 8)
    zeros = None
    if zp != "none":
        zeros = rng.integers(0, 256, size=(rows, zrow), dtype=np.int16).astype(np.uint8)
        zeros = zeros.view(np.int8) if zp == "s8" else zeros
    return data, scales, zeros


def signed_oracle(bits, data, idx, scales, zeros, t):
    """oracle.gather_block_quantized with the type T named (the oracle tells f32 and f16 arrays
    apart by dtype; bf16 values travel as float32)."""
    q = o.as_type(o.unpack_signed(np.take(data, idx, axis=0), bits), t)
    shape = q.shape[:-1] + (scales.shape[-1],)
    zp = None if zeros is None else np.take(zeros, idx, axis=0)
    zero = o.block_zero_points(zp, shape, bits, t, signed=True)
    return o.dequantize(q, zero, o.as_type(np.take(scales, idx, axis=0).astype(np.float32), t), t)


@pytest.mark.parametrize("bits,bs,k,rows,zp,st", SIGNED)
def test_gather_signed_data_bit_exact(bits, bs, k, rows, zp, st):
    """GatherBlockQuantized over s8 data (quantized.ex:49-66 with the sign extension of
    :294-300 and the signed zero-point default of :306-310), bit for bit against the oracle."""
    data, scales, zeros = signed_table(bits, bs, k, rows, zp, st, seed=bits * 1000 + k + rows)
    attrs = {"bits": bits, "block_size": bs, "gather_axis": 0, "quantize_axis": 1}
    idx = np.array([rows - 1, 0, 3, 3, rows // 2, 1], dtype=np.int64)
    names = ["data", "indices", "scales"] + (["zp"] if zeros is not None else [])
    node = Node("GatherBlockQuantized", attrs, names)
    (y,) = quantized.apply(node, [to_dev(data), to_dev(idx), to_dev(scales, st), to_dev(zeros)])
    want = signed_oracle(bits, data, idx, scales, zeros, st)
    if st != "bf16":  # the oracle's own entry point agrees where it can name the type
        np.testing.assert_array_equal(want, o.gather_block_quantized(attrs, data, idx, scales, zeros))
    got = y.float().cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), np.asarray(want, np.float32).view(np.uint32))
    assert device_status() == 0


@pytest.mark.parametrize("bits,zp", [(4, "none"), (4, "u8"), (4, "s8"), (2, "s8"), (8, "u8")])
def test_matmul_over_signed_table(bits, zp):
    """A signed handle multiplies like its dequantized rows (the stored form is the unsigned
    data with flipped top bits and raised zero points): M = 1 and M = 40 within 1e-3."""
    k, rows, bs = 512, 96, 32
    data, scales, zeros = signed_table(bits, bs, k, rows, zp, "f32", seed=7 + bits)
    w = PackedWeight((k, rows, bits, bs), to_dev(data), to_dev(scales), to_dev(zeros), dtype=torch.float32,
                     device=DEV, signed_data=True)
    table = signed_oracle(bits, data, np.arange(rows), scales, zeros, "f32").astype(np.float64)
    np.testing.assert_array_equal(as_np32(w.dequantize()).view(np.uint32),
                                  table.astype(np.float32).view(np.uint32))
    a = np.random.default_rng(3).standard_normal((40, k)).astype(np.float32)
    for m in (1, 40):
        y = as_np32(w.matmul(to_dev(a[:m])))
        assert o.rel_l2(y, a[:m].astype(np.float64) @ table.T) < 1e-3
    w.close()
    assert device_status() == 0
