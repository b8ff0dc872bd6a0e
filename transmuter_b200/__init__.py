"""transmuter_b200: a B200-native (sm_100a) MatMulNBits for Transmuter.

The product is the C-ABI library ``libtq4.so`` (include/tq4.h) with hand-written CUDA kernels;
this package is its Python host side: ``quantized`` mirrors the reference's operator contract
(``Transmuter.Ops.Quantized.apply/2``) and ``sharded`` the N-sharded multi-GPU path.
"""

from . import _lib  # noqa: F401
from .quantized import ArgumentError, Node, PackedWeight, apply, move_weight, packable  # noqa: F401
