"""GPU tests of weights read from ONNX external data (tq4_weight_create_from): the handle made
from file ranges is the handle made from the same bytes in memory, bit for bit, as the
reference's test of a deferred B asserts for its packed weight (test/transmuter/ops_test.exs
:95-117: "The same B in an external file ... packs the same")."""

import numpy as np
import pytest
import torch

from oracle import matmul_nbits as o
from tests.golden_cases import matmul_nbits_cases
from transmuter_b200 import _lib, quantized, workloads
from transmuter_b200.deferred import DeferredTensor, TensorProto
from transmuter_b200.quantized import Node, PackedWeight

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
ONNX = {np.dtype(np.uint8): 2, np.dtype(np.float32): 1, np.dtype(np.float16): 10}


def write_external(dir, arrays, gap=3, last_without_length=True):
    """Writes the arrays one after another (with `gap` filler bytes before each) into dir/data
    and returns a deferred tensor for each, as an exporter's external data entries give them."""
    blob = bytearray()
    out = []
    for i, (name, arr) in enumerate(arrays):
        if arr is None:
            out.append(None)
            continue
        blob += b"\x5a" * gap
        entries = [("location", "data"), ("offset", str(len(blob)))]
        if not (last_without_length and i == len(arrays) - 1):
            entries.append(("length", str(arr.nbytes)))
        blob += np.ascontiguousarray(arr).tobytes()
        proto = TensorProto(name, list(arr.shape), ONNX[arr.dtype], "EXTERNAL", entries)
        out.append(DeferredTensor.new(proto, str(dir)))
    (dir / "data").write_bytes(bytes(blob))
    return out


def bits_of(t):
    return t.float().cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("case", matmul_nbits_cases(), ids=lambda c: c["name"])
def test_fixture_weight_from_external_data(case, tmp_path):
    a, b, scales, zp = (case["inputs"] + [None] * 4)[:4]
    bias = (case["inputs"] + [None] * 6)[5]
    k, n, bits, bs = o.nbits_sizes(case["attrs"])
    node = Node("MatMulNBits", case["attrs"], case["input_names"])
    arrays = [("B", b), ("scales", scales)] + ([("zero_points", zp)] if zp is not None else [])
    ext = write_external(tmp_path, arrays)
    from_file = quantized.move_weight(node, *ext, device=DEV)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)) if x is not None else None
    in_memory = quantized.move_weight(node, t(b), t(scales), t(zp), device=DEV)
    np.testing.assert_array_equal(bits_of(from_file.dequantize()), bits_of(in_memory.dequantize()))
    want = o.dequantize_weight(b, scales, zp, k, n, bits, bs, "f32")
    np.testing.assert_array_equal(bits_of(from_file.dequantize()), want.view(np.uint32))
    y = from_file.matmul(torch.from_numpy(a).to(DEV), torch.from_numpy(bias).to(DEV) if bias is not None else None)
    diff, tol = o.within_reference_tolerance(y.float().cpu().numpy(), case["Y"])
    assert diff <= tol, (diff, tol)


@pytest.mark.parametrize("name,k,n,zp,st", [
    # the C3 lm_head: 77.8 MB of B, 10 chunks over several reader threads, a ragged last chunk
    ("c3-lm-head", 1024, 151936, "none", "f32"),
    # a Llama projection with packed zero points and f16 scales
    ("c5-down", 14336, 4096, "packed", "f16"),
])
def test_large_weight_from_external_data(name, k, n, zp, st, tmp_path):
    cfg = workloads.Config(name, k, n, 1, bits=4, block_size=32 if name.startswith("c3") else 128,
                           scale_type=st, zp=zp)
    p = workloads.make(cfg)
    arrays = [("B", p["B"]), ("scales", p["scales"])] + ([("zero_points", p["zp"])] if p["zp"] is not None else [])
    ext = write_external(tmp_path, arrays, gap=4096 + 5)
    attrs = (cfg.k, cfg.n, cfg.bits, cfg.block_size)
    from_file = PackedWeight(attrs, *ext, device=DEV)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)) if x is not None else None
    in_memory = PackedWeight(attrs, t(p["B"]), t(p["scales"]), t(p["zp"]), device=DEV)
    assert torch.equal(from_file.dequantize(), in_memory.dequantize())
    a = torch.randn(3, cfg.k, device=DEV, dtype=torch.float16)
    assert torch.equal(from_file.matmul(a), in_memory.matmul(a))


def test_mixed_sources(tmp_path):
    """B from the file, scales in host memory, zero points in device memory."""
    cfg = workloads.Config("mixed", 320, 48, 1, bits=4, block_size=64, scale_type="f16", zp="packed")
    p = workloads.make(cfg)
    (b,) = write_external(tmp_path, [("B", p["B"])], gap=1)
    attrs = (cfg.k, cfg.n, cfg.bits, cfg.block_size)
    scales = torch.from_numpy(p["scales"])
    zp = torch.from_numpy(p["zp"]).to(DEV)
    w = PackedWeight(attrs, b, scales, zp, device=DEV)
    want = o.dequantize_weight(p["B"], p["scales"], p["zp"], cfg.k, cfg.n, 4, 64, "f16")
    np.testing.assert_array_equal(w.dequantize().cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_file_range_past_the_end_leaves_no_handle(tmp_path):
    cfg = workloads.Config("short", 64, 16, 1, bits=4, block_size=16, scale_type="f32", zp="none")
    p = workloads.make(cfg)
    b, s = write_external(tmp_path, [("B", p["B"]), ("scales", p["scales"])], last_without_length=False)
    data = tmp_path / "data"
    data.write_bytes(data.read_bytes()[:-1])
    with pytest.raises(_lib.Tq4Error, match="past the end"):
        PackedWeight((cfg.k, cfg.n, 4, 16), b, s, device=DEV)
    torch.cuda.synchronize()
