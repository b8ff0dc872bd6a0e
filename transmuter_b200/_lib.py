"""ctypes binding of libtq4 (include/tq4.h). This is the same surface an Erlang NIF binds.

Loading fails loudly: there is no CPU fallback anywhere in the product path.
"""

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtq4.so")

TQ4_OK = 0
STATUS = {
    0: "ok", 1: "invalid argument", 2: "unsupported", 3: "CUDA error", 4: "NCCL error",
    5: "out of device memory", 6: "timed out", 7: "device-side error", 8: "file error",
}
F32, F16, BF16, U8, S8 = 0, 1, 2, 3, 4
ZP_NONE, ZP_PACKED, ZP_FLOAT = 0, 1, 2
UNIQUE_ID_BYTES = 128

# Every symbol include/tq4.h declares (the CPU tests check the library exports each one).
EXPORTS = [
    "tq4_weight_input_sizes", "tq4_weight_create", "tq4_weight_create_from", "tq4_weight_destroy", "tq4_weight_merge",
    "tq4_weight_info",
    "tq4_matmul", "tq4_matmul_noalloc", "tq4_dequantize", "tq4_gather_rows", "tq4_device_status",
    "tq4_set_wait_limit", "tq4_selftest_peer_wait", "tq4_last_error",
    "tq4_status_string", "tq4_comm_unique_id", "tq4_comm_create", "tq4_comm_destroy",
    "tq4_sharded_create", "tq4_sharded_create_from", "tq4_sharded_rows", "tq4_sharded_matmul", "tq4_sharded_destroy",
    # include/tq4_decoder.h
    "tq4_add_rmsnorm", "tq4_qk_norm_rope", "tq4_attention_decode", "tq4_attention_decode_rope",
    "tq4_matmul_fused", "tq4_silu_mul", "tq4_argmax_advance",
]


class WeightDesc(ctypes.Structure):
    _fields_ = [
        ("K", ctypes.c_int64), ("N", ctypes.c_int64), ("bits", ctypes.c_int32),
        ("block_size", ctypes.c_int32), ("scale_dtype", ctypes.c_int), ("zp_kind", ctypes.c_int),
        ("zp_dtype", ctypes.c_int), ("dequant_dtype", ctypes.c_int), ("b_signed", ctypes.c_int32),
    ]


class Source(ctypes.Structure):
    """``tq4_source``: bytes in memory (``data``), or ``length`` bytes of the file ``path`` from
    ``offset`` (-1: to the end of the file)."""
    _fields_ = [
        ("data", ctypes.c_void_p), ("path", ctypes.c_char_p), ("offset", ctypes.c_int64),
        ("length", ctypes.c_int64),
    ]


class Tq4Error(RuntimeError):
    """A tq4 call returned a non-zero status."""

    def __init__(self, status, message):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status
        self.message = message


_lib = None
_lock = threading.Lock()


def load():
    """Loads libtq4.so (built by ``transmuter_b200.build``). Raises if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libtq4.so is not built ({LIB_PATH}); run python -m transmuter_b200.build")
        lib = ctypes.CDLL(LIB_PATH)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        P = ctypes.POINTER
        sig = {
            "tq4_weight_input_sizes": [P(WeightDesc), P(i64), P(i64), P(i64)],
            "tq4_weight_create": [P(WeightDesc), vp, i64, vp, vp, ctypes.c_int, P(vp)],
            "tq4_weight_create_from": [P(WeightDesc), P(Source), P(Source), P(Source), ctypes.c_int, P(vp)],
            "tq4_weight_destroy": [vp],
            "tq4_weight_merge": [P(vp), ctypes.c_int, P(vp)],
            "tq4_weight_info": [vp, P(WeightDesc), P(i64)],
            "tq4_matmul": [vp, vp, i64, ctypes.c_int, vp, ctypes.c_int, vp, ctypes.c_int, vp],
            "tq4_matmul_noalloc": [vp, vp, i64, ctypes.c_int, vp, ctypes.c_int, vp, ctypes.c_int, vp],
            "tq4_dequantize": [vp, vp, vp],
            "tq4_gather_rows": [vp, vp, i64, vp, vp],
            "tq4_device_status": [ctypes.c_int, P(i32)],
            "tq4_set_wait_limit": [ctypes.c_int, i64],
            "tq4_selftest_peer_wait": [ctypes.c_int, vp],
            "tq4_comm_unique_id": [ctypes.c_char_p],
            "tq4_comm_create": [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P(vp)],
            "tq4_comm_destroy": [vp],
            "tq4_sharded_create": [P(WeightDesc), vp, i64, vp, vp, vp, P(vp)],
            "tq4_sharded_create_from": [P(WeightDesc), P(Source), P(Source), P(Source), vp, P(vp)],
            "tq4_sharded_rows": [vp, P(i64), P(i64)],
            "tq4_sharded_matmul": [vp, vp, i64, ctypes.c_int, vp, ctypes.c_int, vp, ctypes.c_int, vp],
            "tq4_sharded_destroy": [vp],
        }
        for name, args in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        lib.tq4_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        lib.tq4_last_error.restype = ctypes.c_size_t
        lib.tq4_status_string.argtypes = [ctypes.c_int]
        lib.tq4_status_string.restype = ctypes.c_char_p
        _lib = lib
        return lib


def last_error():
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.tq4_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status):
    if status != TQ4_OK:
        raise Tq4Error(status, last_error())
