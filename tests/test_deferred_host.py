"""CPU tests of external initializers (ONNX external data): the mirror of
Transmuter.DeferredTensor and Ops.read_external/2, and the file checks of
tq4_weight_create_from, which all run before any device work."""

import ctypes
import os

import numpy as np
import pytest
import torch

from transmuter_b200 import _lib, deferred, quantized
from transmuter_b200.deferred import DeferredTensor, TensorProto
from transmuter_b200.quantized import ArgumentError, Node, PackedWeight


def external(name, dims, data_type, location, offset=None, length=None):
    entries = [("location", location)]
    if offset is not None:
        entries.append(("offset", str(offset)))
    if length is not None:
        entries.append(("length", str(length)))
    return TensorProto(name, list(dims), data_type, "EXTERNAL", entries)


def test_shape_type_follows_the_reference():
    """Ops.tensor_shape_type/1 (ops.ex:610-627)."""
    assert deferred.tensor_shape_type(TensorProto("s", [2], 8)) is None
    assert deferred.tensor_shape_type(TensorProto("e", [0, 4], 1)) is None
    assert deferred.tensor_shape_type(TensorProto("q", [3, 5], 21)) == ((3, 3), torch.uint8)
    assert deferred.tensor_shape_type(TensorProto("q", [3, 5], 22)) == ((3, 3), torch.int8)
    assert deferred.tensor_shape_type(TensorProto("h", [4, 2], 10)) == ((4, 2), torch.float16)
    assert deferred.tensor_shape_type(TensorProto("b", [7], 16)) == ((7,), torch.bfloat16)


def test_new_defers_only_external_tensors(tmp_path):
    """DeferredTensor.new/2 (deferred_tensor.ex:16-23)."""
    assert DeferredTensor.new(TensorProto("B", [4, 2, 16], 2), str(tmp_path)) is None
    assert DeferredTensor.new(external("s", [0], 1, "data"), str(tmp_path)) is None
    t = DeferredTensor.new(external("B", [4, 2, 16], 2, "data"), str(tmp_path))
    assert (t.shape, t.dtype, t.nbytes) == ((4, 2, 16), torch.uint8, 128)
    assert deferred.shape_type(t) == ((4, 2, 16), torch.uint8)
    assert deferred.shape_type(torch.zeros(3, 2)) == ((3, 2), torch.float32)


def test_value_reads_offset_and_length(tmp_path):
    """read_external/2 (ops.ex:680-695): offset defaults to 0, no length runs to the end."""
    rng = np.random.default_rng(0)
    b = rng.integers(0, 256, 96, dtype=np.uint8)
    s = rng.random(12).astype(np.float16)
    (tmp_path / "data").write_bytes(b"xyz" + b.tobytes() + s.tobytes())
    tb = DeferredTensor.new(external("B", [96], 2, "data", offset=3, length=96), str(tmp_path))
    ts = DeferredTensor.new(external("s", [12], 10, "data", offset=99), str(tmp_path))
    assert np.array_equal(tb.value().numpy(), b)
    assert np.array_equal(ts.value().numpy(), s)
    assert deferred.value(torch.ones(2)).tolist() == [1.0, 1.0]
    assert tb.source() == (str(tmp_path / "data"), 3, 96)
    assert ts.source() == (str(tmp_path / "data"), 99, -1)
    (tmp_path / "head").write_bytes(b.tobytes())
    whole = DeferredTensor.new(external("B", [96], 2, "head"), str(tmp_path))
    assert np.array_equal(whole.value().numpy(), b)
    short = DeferredTensor.new(external("B", [97], 2, "head"), str(tmp_path))
    with pytest.raises(ArgumentError):
        short.value()


def test_packable_reads_a_deferred_shape(tmp_path):
    node = Node("MatMulNBits", {"K": 64, "N": 8, "bits": 4, "block_size": 16}, ["A", "B", "scales"])
    b = DeferredTensor.new(external("B", [8, 4, 8], 2, "data"), str(tmp_path))
    assert quantized.packable(node, b, torch.ones(32))
    wrong = DeferredTensor.new(external("B", [8, 4, 4], 2, "data"), str(tmp_path))
    assert not quantized.packable(node, wrong, torch.ones(32))


# ---- tq4_weight_create_from: the checks before any device work -------------------------------

def desc(K=64, N=8, zk=_lib.ZP_NONE):
    d = _lib.WeightDesc()
    d.K, d.N, d.bits, d.block_size = K, N, 4, 16
    d.scale_dtype, d.zp_kind, d.zp_dtype, d.dequant_dtype = _lib.F32, zk, _lib.U8, _lib.F32
    return d


def file_source(path, offset=0, length=-1):
    s = _lib.Source()
    s.path, s.offset, s.length = str(path).encode(), offset, length
    return s


def mem_source(buf, length):
    s = _lib.Source()
    s.data, s.length = ctypes.addressof(buf), length
    return s


def create_from(d, b, s, z=None):
    h = ctypes.c_void_p()
    st = _lib.load().tq4_weight_create_from(ctypes.byref(d), ctypes.byref(b), ctypes.byref(s),
                                            ctypes.byref(z) if z is not None else None, 0, ctypes.byref(h))
    assert not h.value
    return st, _lib.last_error()


@pytest.fixture
def files(tmp_path):
    # B: 8 rows x 4 blocks x 8 bytes = 256 bytes; scales: 32 f32 = 128 bytes
    (tmp_path / "data").write_bytes(bytes(256) + bytes(128))
    return tmp_path


def test_missing_file_is_an_io_error(files):
    scales = (ctypes.c_uint8 * 128)()
    st, msg = create_from(desc(), file_source(files / "nope"), mem_source(scales, 128))
    assert st == 8 and "nope" in msg and "B" in msg


def test_range_past_the_end_is_rejected(files):
    scales = (ctypes.c_uint8 * 128)()
    st, msg = create_from(desc(), file_source(files / "data", 200, 256), mem_source(scales, 128))
    assert st == 1 and "past the end" in msg


def test_length_must_match_the_description(files):
    scales = (ctypes.c_uint8 * 128)()
    # no length: offset 0 to the end is 384 bytes, B needs 256
    st, msg = create_from(desc(), file_source(files / "data"), mem_source(scales, 128))
    assert st == 1 and "B has 384 bytes" in msg
    st, msg = create_from(desc(), file_source(files / "data", 0, 256), file_source(files / "data", 256, 64))
    assert st == 1 and "scales has 64 bytes" in msg
    st, msg = create_from(desc(), file_source(files / "data", 0, 256), mem_source(scales, 100))
    assert st == 1 and "scales has 100 bytes" in msg


def test_bad_offsets_and_missing_inputs(files):
    scales = (ctypes.c_uint8 * 128)()
    st, msg = create_from(desc(), file_source(files / "data", -1, 256), mem_source(scales, 128))
    assert st == 1 and "offset -1" in msg
    st, msg = create_from(desc(), file_source(files / "data", 0, -2), mem_source(scales, 128))
    assert st == 1
    st, msg = create_from(desc(), file_source(files, 0, 256), mem_source(scales, 128))
    assert st == 8 and "not a regular file" in msg
    st, msg = create_from(desc(zk=_lib.ZP_PACKED), file_source(files / "data", 0, 256), mem_source(scales, 128))
    assert st == 1 and "zero points" in msg
    st, msg = create_from(desc(), _lib.Source(), mem_source(scales, 128))
    assert st == 1 and "B is required" in msg


def test_packed_weight_checks_deferred_sizes_before_the_device(files):
    d = str(files)
    b = DeferredTensor.new(external("B", [8, 4, 8], 2, "data", 0, 256), d)
    s_bad = DeferredTensor.new(external("s", [31], 1, "data", 256, 124), d)
    with pytest.raises(ArgumentError, match="scales have 124 bytes"):
        PackedWeight((64, 8, 4, 16), b, s_bad, device="cuda:0")
    # the sizes agree with the description but the file is too short: the library says so
    s_far = DeferredTensor.new(external("s", [32], 1, "data", 300, 128), d)
    with pytest.raises(_lib.Tq4Error, match="past the end"):
        PackedWeight((64, 8, 4, 16), b, s_far, device="cuda:0")
    assert os.path.getsize(files / "data") == 384


def test_sharded_create_from_checks_arguments():
    lib = _lib.load()
    h = ctypes.c_void_p()
    assert lib.tq4_sharded_create_from(None, None, None, None, None, ctypes.byref(h)) == 1
    assert "null argument" in _lib.last_error() and not h.value
