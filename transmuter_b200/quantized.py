"""Host side of the MatMulNBits hot path: a Python mirror of the reference's operator contract
over the tq4 C ABI, with torch used only for device memory and streams.

Reference interface (georgeguimaraes/transmuter 2.0.0):
- ``Transmuter.Ops.Quantized.apply(node, inputs)`` (lib/transmuter/ops/quantized.ex:27): the
  node's attributes are read with ``attr/3`` (lib/transmuter/ops.ex:582), the positional inputs
  are ``[A, B, scales, zero_points?, g_idx?, bias?]`` with missing optionals as ``nil``
  (ops.ex:446), and the result is a list of outputs.
- ``Transmuter.move/2`` (lib/transmuter.ex:1104-1182) gives each packable MatMulNBits node a
  weight built once at load (``dequantized_weight/6`` at :1230-1240; the EMLX packer
  lib/transmuter/emlx.ex:104-148 is the precedent for a backend-owned packed weight). Here the
  weight is a ``PackedWeight``: a tq4 handle that keeps B packed on the GPU.

B, scales and zero points may be ``DeferredTensor`` values (initializers in an ONNX external
data file, ``deferred.py``): the weight then reads their file ranges straight to the GPU.

Errors follow the reference: unsupported inputs raise ``ArgumentError`` (quantized.ex:33-34).
"""

import ctypes
import math
from dataclasses import dataclass, field

import torch

from . import _lib
from .deferred import ArgumentError, DeferredTensor, shape_type

TORCH_TO_TQ4 = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.uint8: _lib.U8,
                torch.int8: _lib.S8}
TQ4_TO_TORCH = {v: k for k, v in TORCH_TO_TQ4.items()}
NAME_TO_TORCH = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@dataclass
class Node:
    """The parts of an ONNX NodeProto the operator reads (``%Transmuter.Onnx.NodeProto{}``)."""
    op_type: str
    attribute: dict = field(default_factory=dict)
    input: list = field(default_factory=list)
    output: list = field(default_factory=lambda: ["Y"])
    name: str = ""


def attr(node, name, default=None):
    """``Ops.attr/3`` (ops.ex:582)."""
    return node.attribute.get(name, default)


def optional(inputs, count):
    """``Ops.optional/2`` (ops.ex:446): pads the optional inputs with None."""
    return (list(inputs) + [None] * count)[:count]


def nbits_sizes(node):
    """``Quantized.nbits_sizes/1`` (quantized.ex:226-228). ``accuracy_level`` is ignored, as in
    the reference."""
    k, n, bits, bs = attr(node, "K"), attr(node, "N"), attr(node, "bits", 4), attr(node, "block_size")
    if k is None or n is None or bs is None:
        raise ArgumentError("MatMulNBits needs the K, N and block_size attributes")
    return int(k), int(n), int(bits), int(bs)


def merge_type(a, b):
    """Nx type promotion of two float types (f16 with bf16 gives f32)."""
    return a if a == b else torch.float32


def upcast(dtype, compute_type):
    """``Transmuter.upcast/2`` (lib/transmuter.ex:1323-1327) on a dtype."""
    if compute_type is not None and dtype in (torch.float16, torch.bfloat16):
        return compute_type
    return dtype


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _nbytes(x):
    if isinstance(x, DeferredTensor):
        return x.nbytes
    return x.numel() * x.element_size()


def _source(x, nbytes):
    """A ``tq4_source`` for a tensor (its memory) or a deferred tensor (its file range)."""
    src = _lib.Source()
    if isinstance(x, DeferredTensor):
        path, offset, length = x.source()
        src.path, src.offset, src.length = path.encode(), offset, length
    else:
        src.data, src.length = x.data_ptr(), nbytes
    return src


class PackedWeight:
    """A MatMulNBits weight held packed on one GPU by a tq4 handle (the "B:packed" value of a
    moved model). ``dtype`` is the type T it dequantizes in. ``signed_data`` takes s8 data (a
    GatherBlockQuantized table of an int4 export; MatMulNBits' B is always u8): its values are
    sign extended and the default zero point is 0 (quantized.ex:294-325)."""

    def __init__(self, attrs, b, scales, zero_points=None, dtype=None, device=None, signed_data=False):
        k, n, bits, bs = attrs
        self.k, self.n, self.bits, self.block_size = k, n, bits, bs
        b_type, s_type = shape_type(b)[1], shape_type(scales)[1]
        z_type = shape_type(zero_points)[1] if zero_points is not None else None
        if b_type != (torch.int8 if signed_data else torch.uint8):
            raise ArgumentError(f"MatMulNBits B must be {'s8' if signed_data else 'u8'}, got {b_type}")
        if s_type not in (torch.float32, torch.float16, torch.bfloat16):
            raise ArgumentError(f"MatMulNBits scales must be a float tensor, got {s_type}")
        self.dtype = dtype or s_type
        desc = _lib.WeightDesc()
        desc.K, desc.N, desc.bits, desc.block_size = k, n, bits, bs
        desc.scale_dtype = TORCH_TO_TQ4[s_type]
        desc.dequant_dtype = TORCH_TO_TQ4[self.dtype]
        desc.b_signed = 1 if signed_data else 0
        if zero_points is None:
            desc.zp_kind, desc.zp_dtype = _lib.ZP_NONE, _lib.U8
        elif z_type in (torch.uint8, torch.int8):
            desc.zp_kind, desc.zp_dtype = _lib.ZP_PACKED, TORCH_TO_TQ4[z_type]
        elif z_type in (torch.float32, torch.float16, torch.bfloat16):
            desc.zp_kind, desc.zp_dtype = _lib.ZP_FLOAT, TORCH_TO_TQ4[z_type]
        else:
            raise ArgumentError(f"MatMulNBits zero points must be u8, s8 or float, got {z_type}")
        self.desc = desc
        if device is None:
            device = b.device if isinstance(b, torch.Tensor) and b.is_cuda else torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        lib = _lib.load()
        sizes = [ctypes.c_int64() for _ in range(3)]
        _lib.check(lib.tq4_weight_input_sizes(ctypes.byref(desc), *[ctypes.byref(s) for s in sizes]))
        b_bytes, s_bytes, z_bytes = (s.value for s in sizes)
        inputs = [x if isinstance(x, DeferredTensor) else x.contiguous() for x in (b, scales)]
        if zero_points is not None:
            inputs.append(zero_points if isinstance(zero_points, DeferredTensor) else zero_points.contiguous())
        got = [_nbytes(x) for x in inputs]
        if got[0] != b_bytes:
            raise ArgumentError(f"MatMulNBits B has {got[0]} bytes, expected {b_bytes}")
        if got[1] != s_bytes:
            raise ArgumentError(f"MatMulNBits scales have {got[1]} bytes, expected {s_bytes}")
        if zero_points is not None and got[2] != z_bytes:
            raise ArgumentError(f"MatMulNBits zero points have {got[2]} bytes, expected {z_bytes}")
        handle = ctypes.c_void_p()
        if any(isinstance(x, DeferredTensor) for x in inputs):
            sources = [_source(x, nb) for x, nb in zip(inputs, got)]
            _lib.check(lib.tq4_weight_create_from(
                ctypes.byref(desc), ctypes.byref(sources[0]), ctypes.byref(sources[1]),
                ctypes.byref(sources[2]) if zero_points is not None else None,
                self.device.index or 0, ctypes.byref(handle)))
        else:
            _lib.check(lib.tq4_weight_create(
                ctypes.byref(desc), _ptr(inputs[0]), b_bytes, _ptr(inputs[1]),
                _ptr(inputs[2]) if zero_points is not None else None, self.device.index or 0,
                ctypes.byref(handle)))
        self._handle = handle
        self._lib = lib

    @classmethod
    def merge(cls, parts):
        """One weight over the rows of ``parts`` in order (``tq4_weight_merge``; the packed form of
        ``Fusion.matmuls/2``, lib/transmuter/fusion.ex:430-540). The parts stay valid."""
        if not parts:
            raise ArgumentError("merge needs at least one weight")
        lib = _lib.load()
        arr = (ctypes.c_void_p * len(parts))(*[p._handle.value for p in parts])
        handle = ctypes.c_void_p()
        _lib.check(lib.tq4_weight_merge(arr, len(parts), ctypes.byref(handle)))
        w = cls.__new__(cls)
        first = parts[0]
        w.k, w.bits, w.block_size = first.k, first.bits, first.block_size
        w.n = sum(p.n for p in parts)
        w.dtype, w.device, w._lib, w._handle = first.dtype, first.device, lib, handle
        w.desc = _lib.WeightDesc()
        ctypes.memmove(ctypes.byref(w.desc), ctypes.byref(first.desc), ctypes.sizeof(_lib.WeightDesc))
        w.desc.N = w.n
        return w

    @property
    def shape(self):
        return (self.n, self.k)

    def close(self):
        if getattr(self, "_handle", None):
            self._lib.tq4_weight_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def matmul(self, a, bias=None, out_dtype=None, out=None):
        """Y = A . W^T (+ bias) over the last axis of A (a CUDA tensor on the handle's device)."""
        if not a.is_cuda:
            raise ArgumentError("MatMulNBits A must be a CUDA tensor on the weight's device")
        if a.shape[-1] != self.k:
            raise ArgumentError(f"MatMulNBits A has {a.shape[-1]} columns, expected K={self.k}")
        if a.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ArgumentError(f"MatMulNBits A must be f32, f16 or bf16, got {a.dtype}")
        lead = a.shape[:-1]
        a2 = a.reshape(-1, self.k).contiguous()
        m = a2.shape[0]
        out_dtype = out_dtype or merge_type(a.dtype, self.dtype)
        if bias is not None:
            if bias.numel() != self.n:
                raise ArgumentError(f"MatMulNBits bias has {bias.numel()} values, expected N={self.n}")
            bias = bias.contiguous()
            out_dtype = merge_type(out_dtype, bias.dtype)
        y = out if out is not None else torch.empty((m, self.n), dtype=out_dtype, device=a.device)
        _lib.check(self._lib.tq4_matmul(
            self._handle, _ptr(a2), m, TORCH_TO_TQ4[a2.dtype], _ptr(bias),
            TORCH_TO_TQ4[bias.dtype] if bias is not None else 0, _ptr(y), TORCH_TO_TQ4[y.dtype],
            _stream(a.device)))
        return y.reshape(*lead, self.n)

    def dequantize(self):
        """``dequantize_weight/4`` (quantized.ex:234-240): W {N, K} in ``self.dtype``, bit-exact."""
        w = torch.empty((self.n, self.k), dtype=self.dtype, device=self.device)
        _lib.check(self._lib.tq4_dequantize(self._handle, _ptr(w), _stream(self.device)))
        return w

    def gather(self, indices):
        """Dequantized rows ``indices`` (GatherBlockQuantized, quantized.ex:49-66)."""
        idx = indices.to(device=self.device, dtype=torch.int64).contiguous()
        out = torch.empty((*idx.shape, self.k), dtype=self.dtype, device=self.device)
        _lib.check(self._lib.tq4_gather_rows(self._handle, _ptr(idx), idx.numel(), _ptr(out), _stream(self.device)))
        return out


def packable(node, b, scales, g_idx=None):
    """``packable?/2`` (lib/transmuter.ex:1209-1225), widened: a K that is not a multiple of
    block_size is packable too (its B rows hold whole padded blocks)."""
    if node.op_type != "MatMulNBits" or scales is None or g_idx is not None or b is None:
        return False
    k, n, bits, bs = nbits_sizes(node)
    blocks = -(-k // bs)
    # packed_bytes?/2 (lib/transmuter.ex:1219-1226) reads the shape and type of a tensor or of a
    # deferred one without reading its data
    shape, dtype = shape_type(b)
    return bits in (2, 4, 8) and dtype == torch.uint8 and math.prod(shape) == n * blocks * bs * bits // 8


def move_weight(node, b, scales, zero_points=None, compute_type=None, device=None):
    """The weight ``move/2`` builds for one node (lib/transmuter.ex:1155-1164,1230-1240), in the
    scales' type after ``compute_type``. B, scales and zero points may be deferred tensors."""
    dtype = upcast(shape_type(scales)[1], compute_type)
    return PackedWeight(nbits_sizes(node), b, scales, zero_points, dtype=dtype, device=device)


def apply(node, inputs):
    """``Quantized.apply/2`` for MatMulNBits and GatherBlockQuantized: returns a list."""
    return [op(node, list(inputs))]


def op(node, inputs):
    if node.op_type == "MatMulNBits":
        a, b, scales, *rest = inputs + [None] * max(0, 3 - len(inputs))
        zero_points, g_idx, bias = optional(rest, 3)
        if g_idx is not None:
            raise ArgumentError("MatMulNBits with the g_idx input is not supported")
        k, n, bits, bs = nbits_sizes(node)
        if isinstance(b, PackedWeight):
            # a moved model: the weight was built at load (quantized.ex:39-41)
            return b.matmul(a, bias)
        if b.dtype != torch.uint8 and tuple(b.shape) == (n, k):
            # a float {N, K} weight needs no unpacking (quantized.ex:39-41): a plain matmul
            y = torch.matmul(a, b.t())
            return y + bias if bias is not None else y
        # in the graph: dequantize in A's type on each call (quantized.ex:42)
        w = PackedWeight((k, n, bits, bs), b, scales, zero_points, dtype=a.dtype, device=a.device)
        try:
            return w.matmul(a, bias)
        finally:
            w.close()
    if node.op_type == "GatherBlockQuantized":
        data, indices, scales, *rest = inputs
        zero_points = rest[0] if rest else None
        rank = data.dim()
        qa = attr(node, "quantize_axis", 1)
        if attr(node, "gather_axis", 0) != 0 or (qa % rank if qa is not None else rank - 1) != rank - 1:
            raise ArgumentError("GatherBlockQuantized supports gather_axis 0 and quantize_axis on the last axis")
        if data.dtype not in (torch.uint8, torch.int8) or rank != 2:
            raise ArgumentError("GatherBlockQuantized supports u8 or s8 data of rank 2")
        bits = attr(node, "bits", 4)
        bs = attr(node, "block_size", 128)
        rows, cols = data.shape
        k = cols * 8 // bits
        blocks = scales.shape[-1]
        if blocks * bs < k or -(-k // bs) != blocks:
            raise ArgumentError("GatherBlockQuantized: scales do not match the data and block_size")
        # the table as a MatMulNBits weight: rows of B are rows of the table (same bit order)
        w = PackedWeight((k, rows, bits, bs), data.reshape(-1), scales.reshape(-1),
                         zero_points.reshape(-1) if zero_points is not None else None,
                         dtype=scales.dtype, device=indices.device if indices.is_cuda else None,
                         signed_data=data.dtype == torch.int8)
        try:
            return w.gather(indices)
        finally:
            w.close()
    raise ArgumentError(f"unsupported operator {node.op_type}")
