"""N-sharded MatMulNBits across GPUs (one process per GPU): the Python side of
``tq4_comm_*`` / ``tq4_sharded_*`` (include/tq4.h).

Each rank owns ``share`` = ceil(N/P) rounded up to 16 rows of B, scales and zero points, computes
its columns of Y, and an NCCL all-gather over NVLink builds Y on every rank. The row plan below
is the same arithmetic as ``csrc/sharded.cu`` (kept here so the bookkeeping is testable on CPU).
B, scales and zero points may be deferred tensors (ONNX external data): each rank then reads only
its rows of the files (``tq4_sharded_create_from``).
"""

import ctypes

import torch

from . import _lib
from .deferred import DeferredTensor
from .quantized import TORCH_TO_TQ4, ArgumentError, _nbytes, _ptr, _source, _stream


def shard_share(n, nranks):
    """Rows per rank: ceil(N / P) rounded up to a multiple of 16."""
    return (-(-n // nranks) + 15) // 16 * 16


def shard_rows(n, nranks, rank):
    """(first, count) rows of rank ``rank``; count may be 0 for the last ranks of a small N."""
    share = shard_share(n, nranks)
    first = min(n, rank * share)
    return first, min(n - first, share)


def shard_range(offset, total_bytes, n, nranks, rank):
    """(offset, length) of rank ``rank``'s rows within an input of N equal rows stored from
    ``offset`` in a file: the narrowing ``tq4_sharded_create_from`` applies to external data."""
    row = total_bytes // n
    first, count = shard_rows(n, nranks, rank)
    return offset + first * row, count * row


def unshard(gathered, m, n, nranks):
    """[P, M, share] (the all-gather order) -> [M, N]."""
    share = shard_share(n, nranks)
    g = gathered.reshape(nranks, m, share)
    return g.permute(1, 0, 2).reshape(m, nranks * share)[:, :n]


class Comm:
    """An NCCL communicator made by tq4 (non-blocking init with a deadline)."""

    def __init__(self, unique_id, nranks, rank, device, timeout_ms=60000):
        lib = _lib.load()
        handle = ctypes.c_void_p()
        _lib.check(lib.tq4_comm_create(bytes(unique_id), nranks, rank, device, timeout_ms, ctypes.byref(handle)))
        self._handle, self._lib = handle, lib
        self.nranks, self.rank, self.device = nranks, rank, device

    @staticmethod
    def unique_id():
        lib = _lib.load()
        buf = ctypes.create_string_buffer(_lib.UNIQUE_ID_BYTES)
        _lib.check(lib.tq4_comm_unique_id(buf))
        return buf.raw

    def close(self):
        if getattr(self, "_handle", None):
            self._lib.tq4_comm_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ShardedWeight:
    """This rank's rows of a MatMulNBits weight; ``matmul`` returns the full Y on every rank."""

    def __init__(self, comm, attrs, b, scales, zero_points=None, dtype=None):
        k, n, bits, bs = attrs
        desc = _lib.WeightDesc()
        desc.K, desc.N, desc.bits, desc.block_size = k, n, bits, bs
        desc.scale_dtype = TORCH_TO_TQ4[scales.dtype]
        self.dtype = dtype or scales.dtype
        desc.dequant_dtype = TORCH_TO_TQ4[self.dtype]
        if zero_points is None:
            desc.zp_kind, desc.zp_dtype = _lib.ZP_NONE, _lib.U8
        elif zero_points.dtype == torch.uint8:
            desc.zp_kind, desc.zp_dtype = _lib.ZP_PACKED, _lib.U8
        else:
            desc.zp_kind, desc.zp_dtype = _lib.ZP_FLOAT, TORCH_TO_TQ4[zero_points.dtype]
        self.k, self.n, self.comm = k, n, comm
        self.device = torch.device("cuda", comm.device)
        lib = _lib.load()
        handle = ctypes.c_void_p()
        inputs = [b, scales] + ([zero_points] if zero_points is not None else [])
        if any(isinstance(x, DeferredTensor) for x in inputs):
            # ONNX external data: each rank reads only its rows of the files
            sources = [_source(x if isinstance(x, DeferredTensor) else x.contiguous(), _nbytes(x)) for x in inputs]
            _lib.check(lib.tq4_sharded_create_from(
                ctypes.byref(desc), ctypes.byref(sources[0]), ctypes.byref(sources[1]),
                ctypes.byref(sources[2]) if zero_points is not None else None, comm._handle,
                ctypes.byref(handle)))
        else:
            b = b.contiguous()
            scales = scales.contiguous()
            zero_points = zero_points.contiguous() if zero_points is not None else None
            _lib.check(lib.tq4_sharded_create(ctypes.byref(desc), _ptr(b), b.numel(), _ptr(scales),
                                              _ptr(zero_points), comm._handle, ctypes.byref(handle)))
        self._handle, self._lib = handle, lib
        first, count = ctypes.c_int64(), ctypes.c_int64()
        _lib.check(lib.tq4_sharded_rows(handle, ctypes.byref(first), ctypes.byref(count)))
        self.first, self.count = first.value, count.value

    def matmul(self, a, bias=None, out_dtype=None, out=None):
        if a.shape[-1] != self.k:
            raise ArgumentError(f"MatMulNBits A has {a.shape[-1]} columns, expected K={self.k}")
        lead = a.shape[:-1]
        a2 = a.reshape(-1, self.k).contiguous()
        out_dtype = out_dtype or (a.dtype if a.dtype == self.dtype else torch.float32)
        y = out if out is not None else torch.empty((a2.shape[0], self.n), dtype=out_dtype, device=a.device)
        _lib.check(self._lib.tq4_sharded_matmul(
            self._handle, _ptr(a2), a2.shape[0], TORCH_TO_TQ4[a2.dtype], _ptr(bias),
            TORCH_TO_TQ4[bias.dtype] if bias is not None else 0, _ptr(y), TORCH_TO_TQ4[y.dtype],
            _stream(a.device)))
        return y.reshape(*lead, self.n)

    def close(self):
        if getattr(self, "_handle", None):
            self._lib.tq4_sharded_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
