"""CPU tests of the C-ABI library (loads, exports every symbol of include/tq4.h, validates
arguments before touching a GPU) and of the host-side operator logic (the mirror of
Transmuter.Ops.Quantized.apply/2)."""

import ctypes
import os
import re

import pytest
import torch

from transmuter_b200 import _lib, quantized
from transmuter_b200.quantized import ArgumentError, Node

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for header in sorted(os.listdir(inc)):
        if header.endswith(".h"):
            names |= set(re.findall(r"\b(tq4_[a-z_]+)\s*\(", open(os.path.join(inc, header)).read()))
    return sorted(names)


def test_header_and_binding_agree():
    assert header_symbols() == sorted(_lib.EXPORTS)


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    for name in header_symbols():
        assert hasattr(lib, name), name


def desc(**kw):
    d = _lib.WeightDesc()
    d.K, d.N, d.bits, d.block_size = kw.get("K", 1024), kw.get("N", 3072), kw.get("bits", 4), kw.get("bs", 32)
    d.scale_dtype, d.zp_kind, d.zp_dtype = kw.get("st", _lib.F32), kw.get("zk", _lib.ZP_NONE), kw.get("zt", _lib.U8)
    d.dequant_dtype = kw.get("dt", _lib.F32)
    d.b_signed = kw.get("signed", 0)
    return d


def sizes(d):
    lib = _lib.load()
    out = [ctypes.c_int64() for _ in range(3)]
    st = lib.tq4_weight_input_sizes(ctypes.byref(d), *[ctypes.byref(x) for x in out])
    return st, [x.value for x in out]


def test_signed_data_descriptions():
    """s8 data (GatherBlockQuantized tables of int4 exports) with no, u8 or s8 packed zero points
    has the sizes of u8 data."""
    for zk, zt in ((_lib.ZP_NONE, _lib.U8), (_lib.ZP_PACKED, _lib.U8), (_lib.ZP_PACKED, _lib.S8)):
        for bits in (2, 4, 8):
            st, got = sizes(desc(K=64, N=8, bits=bits, signed=1, zk=zk, zt=zt))
            assert st == 0, _lib.last_error()
            assert got == sizes(desc(K=64, N=8, bits=bits, zk=zk, zt=zt))[1]
    st, _ = sizes(desc(signed=1, bits=8, zk=_lib.ZP_PACKED, zt=_lib.S8, dt=_lib.BF16))
    assert st == 0  # s8 zero points stay within bf16's exact integers


def test_input_sizes():
    st, (b, s, z) = sizes(desc())
    assert st == 0 and (b, s, z) == (3072 * 32 * 16, 3072 * 32 * 4, 0)
    st, (b, s, z) = sizes(desc(K=72, N=16, zk=_lib.ZP_PACKED, st=_lib.F16))
    assert st == 0 and (b, s, z) == (16 * 3 * 16, 16 * 3 * 2, 16 * 2)  # K tail padded to 3 blocks
    st, (b, s, z) = sizes(desc(K=64, N=8, bits=2, bs=16, zk=_lib.ZP_FLOAT, zt=_lib.F32))
    assert st == 0 and (b, s, z) == (8 * 4 * 4, 8 * 4 * 4, 8 * 4 * 4)


@pytest.mark.parametrize("kw,status,msg", [
    ({"bits": 3}, 2, "bits"), ({"bs": 24}, 1, "block_size"), ({"bs": 8}, 1, "block_size"),
    ({"K": 0}, 1, "positive"), ({"zk": _lib.ZP_PACKED, "zt": _lib.F32}, 1, "packed zero points"),
    ({"dt": _lib.U8}, 1, "dequantize type"),
    # signed (s8) data: no float zero points; 8 bits with u8 zero points not in bf16
    ({"signed": 2}, 1, "b_signed"), ({"signed": 1, "zk": _lib.ZP_FLOAT, "zt": _lib.F32}, 2, "float zero points"),
    ({"signed": 1, "bits": 8, "zk": _lib.ZP_PACKED, "zt": _lib.U8, "dt": _lib.BF16}, 2, "bf16"),
])
def test_bad_attributes_return_status(kw, status, msg):
    st, _ = sizes(desc(**kw))
    assert st == status
    assert msg in _lib.last_error()


def test_create_rejects_wrong_b_size_without_a_gpu():
    lib = _lib.load()
    d = desc(K=64, N=8)
    buf = (ctypes.c_uint8 * 10)()
    h = ctypes.c_void_p()
    st = lib.tq4_weight_create(ctypes.byref(d), buf, 10, buf, None, 0, ctypes.byref(h))
    assert st == 1 and "B has 10 bytes" in _lib.last_error() and not h.value


def test_null_handles():
    lib = _lib.load()
    assert lib.tq4_matmul(None, None, 1, 0, None, 0, None, 0, None) == 1
    assert lib.tq4_weight_destroy(None) == 0
    assert lib.tq4_status_string(6) == b"timed out"


# ---- host logic ------------------------------------------------------------------------------

def node(**attrs):
    base = {"K": 64, "N": 8, "bits": 4, "block_size": 16}
    base.update(attrs)
    return Node("MatMulNBits", base, ["A", "B", "scales"])


def test_nbits_sizes_defaults_and_accuracy_level_ignored():
    n = Node("MatMulNBits", {"K": 64, "N": 8, "block_size": 16, "accuracy_level": 4})
    assert quantized.nbits_sizes(n) == (64, 8, 4, 16)
    with pytest.raises(ArgumentError):
        quantized.nbits_sizes(Node("MatMulNBits", {"K": 64}))


def test_optional_pads_with_none():
    assert quantized.optional([1], 3) == [1, None, None]
    assert quantized.optional([], 3) == [None, None, None]


def test_g_idx_raises_argument_error_before_any_device_work():
    a = torch.zeros(1, 64)
    with pytest.raises(ArgumentError, match="g_idx"):
        quantized.apply(node(), [a, torch.zeros(8, 4, 8, dtype=torch.uint8), torch.ones(32), None, torch.zeros(64, dtype=torch.int32)])


def test_unsupported_op_raises():
    with pytest.raises(ArgumentError):
        quantized.apply(Node("QLinearMatMul", {}), [])


def test_dense_weight_passes_through():
    """quantized.ex:39-41: a B already shaped {N, K} is multiplied as is."""
    a = torch.randn(2, 64)
    w = torch.randn(8, 64)
    (y,) = quantized.apply(node(), [a, w, None])
    torch.testing.assert_close(y, a @ w.T)


def test_packable():
    b = torch.zeros(8 * 4 * 8, dtype=torch.uint8)
    assert quantized.packable(node(), b, torch.ones(32))
    assert not quantized.packable(node(), b, None)
    assert not quantized.packable(node(), b, torch.ones(32), g_idx=torch.zeros(1))
    assert not quantized.packable(node(bits=3), b, torch.ones(32))
    # K % block_size != 0 is accepted (the reference leaves such nodes in the graph)
    assert quantized.packable(node(K=72, block_size=32, N=16), torch.zeros(16 * 3 * 16, dtype=torch.uint8), torch.ones(48))


def test_type_promotion_and_upcast():
    assert quantized.merge_type(torch.float16, torch.float16) == torch.float16
    assert quantized.merge_type(torch.float16, torch.bfloat16) == torch.float32
    assert quantized.upcast(torch.float16, torch.float32) == torch.float32
    assert quantized.upcast(torch.float32, torch.float16) == torch.float32
    assert quantized.upcast(torch.float16, None) == torch.float16
