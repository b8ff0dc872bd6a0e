"""Initializers whose data an ONNX model keeps in a file beside it, read at load time.

Reference (georgeguimaraes/transmuter 2.0.0):
- ``Transmuter.DeferredTensor`` (lib/transmuter/deferred_tensor.ex): with a backend, ``load!/2``
  keeps each external initializer as a deferred tensor (lib/transmuter.ex:186-196) that knows its
  shape and type; ``move/2`` reads it with ``value/1`` only when it moves the param
  (lib/transmuter.ex:1159), so the file data of all params is never in memory at once.
- ``Ops.read_external/2`` (lib/transmuter/ops.ex:680-695): the file is the model's directory
  joined with the ``location`` entry; ``offset`` defaults to 0 and a missing ``length`` means
  "to the end of the file".
- ``Ops.tensor_shape_type/1`` (ops.ex:610-627): strings and tensors with a zero dimension have
  no deferred form; 4-bit types stay packed two values per byte.

A ``PackedWeight`` given deferred inputs passes their file ranges to ``tq4_weight_create_from``,
which streams them to the GPU through pinned chunks: the tensor is never whole in host memory.
``value()`` is the host read of the reference, for inputs that are not moved.
"""

import math
import os
from dataclasses import dataclass, field

import numpy as np
import torch

# ONNX TensorProto.DataType -> the element type of the tensor's bytes (ops.ex:700-719).
ONNX_TYPES = {
    1: torch.float32, 2: torch.uint8, 3: torch.int8, 5: torch.int16, 6: torch.int32,
    7: torch.int64, 9: torch.uint8, 10: torch.float16, 11: torch.float64, 16: torch.bfloat16,
}
STRING, UINT4, INT4 = 8, 21, 22
FP8_TYPES = (17, 18, 19, 20)


class ArgumentError(ValueError):
    """The reference's ArgumentError."""


@dataclass
class TensorProto:
    """The fields of an ONNX TensorProto that locate an initializer's data
    (``%Transmuter.Onnx.TensorProto{}``); ``external_data`` holds the StringStringEntryProto
    pairs as (key, value)."""
    name: str
    dims: list
    data_type: int
    data_location: str = "DEFAULT"
    external_data: list = field(default_factory=list)


def tensor_shape_type(proto):
    """``Ops.tensor_shape_type/1`` (ops.ex:610-627): (shape, dtype), or None for a string or an
    empty tensor."""
    if proto.data_type == STRING or 0 in proto.dims:
        return None
    dims = list(proto.dims)
    if proto.data_type in (UINT4, INT4):
        return tuple(dims[:-1] + [(dims[-1] + 1) // 2]), torch.int8 if proto.data_type == INT4 else torch.uint8
    if proto.data_type in FP8_TYPES:
        return tuple(dims), torch.float16
    if proto.data_type not in ONNX_TYPES:
        raise ArgumentError(f"ONNX type {proto.data_type} has no type here")
    return tuple(dims), ONNX_TYPES[proto.data_type]


def external_range(proto, dir):
    """The entries ``Ops.read_external/2`` reads (ops.ex:680-690): (path, offset, length), where
    length is None when the entry is absent (the data runs to the end of the file)."""
    entries = dict(proto.external_data)
    if "location" not in entries:
        raise ArgumentError(f"the external initializer {proto.name} has no location")
    path = os.path.join(dir, entries["location"])
    offset = int(entries.get("offset", "0"))
    length = int(entries["length"]) if "length" in entries else None
    return path, offset, length


@dataclass
class DeferredTensor:
    """``Transmuter.DeferredTensor``: an external initializer read only when it is needed."""
    shape: tuple
    dtype: torch.dtype
    proto: TensorProto
    dir: str

    @staticmethod
    def new(proto, dir):
        """``DeferredTensor.new/2`` (deferred_tensor.ex:16-23): None unless the proto keeps its
        data in a file and has a shape and a type."""
        if proto.data_location != "EXTERNAL":
            return None
        st = tensor_shape_type(proto)
        if st is None:
            return None
        return DeferredTensor(st[0], st[1], proto, dir)

    @property
    def nbytes(self):
        return math.prod(self.shape) * torch.empty((), dtype=self.dtype).element_size()

    def source(self):
        """(path, offset, length or -1) for ``tq4_source``."""
        path, offset, length = external_range(self.proto, self.dir)
        return path, offset, -1 if length is None else length

    def value(self):
        """``DeferredTensor.value/1`` (deferred_tensor.ex:27): the tensor, read on the host."""
        if self.proto.data_type in FP8_TYPES:
            raise ArgumentError("reading fp8 external data is not supported here")
        path, offset, length = external_range(self.proto, self.dir)
        if length is None:
            length = os.stat(path).st_size - offset
        if length != self.nbytes:
            raise ArgumentError(f"the external data of {self.proto.name} has {length} bytes, expected {self.nbytes}")
        with open(path, "rb") as f:
            f.seek(offset)
            raw = f.read(length)
        if len(raw) != length:
            raise ArgumentError(f"{path} ends before the external data of {self.proto.name}")
        arr = np.frombuffer(bytearray(raw), dtype=np.uint8)
        return torch.from_numpy(arr).view(self.dtype).reshape(self.shape)


def value(t):
    """``DeferredTensor.value/1`` of a param: a deferred tensor is read, a tensor is itself."""
    return t.value() if isinstance(t, DeferredTensor) else t


def shape_type(t):
    """``DeferredTensor.shape_type/1`` (deferred_tensor.ex:31-33)."""
    if isinstance(t, DeferredTensor):
        return t.shape, t.dtype
    return tuple(t.shape), t.dtype
