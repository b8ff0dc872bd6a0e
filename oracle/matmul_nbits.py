"""CPU oracle for the com.microsoft MatMulNBits operator: a numpy restatement of the reference's
Nx arithmetic. TEST INFRASTRUCTURE ONLY: the tests, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it as the checker and as the
timed CPU stand-in for the reference. The product path (``transmuter_b200``) never imports it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks this module against the six
MatMulNBits and two GatherBlockQuantized known-answer fixtures that the reference records with
ONNX Runtime (``test/fixtures/ops/MatMulNBits_*``, extracted by ``tests/golden/make_golden.py``).

References are to georgeguimaraes/transmuter 2.0.0:
- ``lib/transmuter/ops/quantized.ex:30-46``   the MatMulNBits clause
- ``lib/transmuter/ops/quantized.ex:49-66``   GatherBlockQuantized
- ``lib/transmuter/ops/quantized.ex:226-228`` ``nbits_sizes/1``
- ``lib/transmuter/ops/quantized.ex:234-240`` ``dequantize_weight/4``
- ``lib/transmuter/ops/quantized.ex:294-325`` sign extension and ``block_zero_points/5``
- ``lib/transmuter/ops/packed.ex:9-36``       ``Packed.unpack/2`` and ``Packed.dequantize/3``
- ``lib/transmuter.ex:1230-1240,1323-1327``   the moved weight and ``upcast/2``

Float types: "f32", "f16" and "bf16". numpy has no bfloat16, so bf16 values are carried as
float32 arrays that hold only bf16-representable numbers (``round_bf16``).
"""

import numpy as np

FLOAT_TYPES = ("f32", "f16", "bf16")


def round_bf16(x):
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(nan, np.float32(np.nan), out)


def round_bf16_from_f64(x):
    """Round float64 values to the nearest bfloat16 with ONE rounding (returned as float32).
    A float32 intermediate may land exactly on a bfloat16 midpoint; those cases are resolved
    from the float64 value."""
    x = np.asarray(x, np.float64)
    y = x.astype(np.float32)
    bits = np.ascontiguousarray(y).view(np.uint32).astype(np.uint64)
    tie = ((bits & 0xFFFF) == 0x8000) & (y.astype(np.float64) != x)
    out = round_bf16(y)
    if tie.any():
        away = np.abs(x) > np.abs(y.astype(np.float64))
        up = (((bits >> 16) + 1) << 16).astype(np.uint32).view(np.float32)
        down = ((bits >> 16) << 16).astype(np.uint32).view(np.float32)
        out = np.where(tie, np.where(away, up, down), out)
    return out.astype(np.float32)


def as_type(x, t):
    """``Nx.as_type`` to a float type: one round-to-nearest-even."""
    if t == "f32":
        return np.asarray(x, dtype=np.float32)
    if t == "f16":
        return np.asarray(x, dtype=np.float16)
    if t == "bf16":
        return round_bf16(np.asarray(x, dtype=np.float32))
    raise ValueError(f"unsupported float type {t}")


def type_of(x):
    """The float type name of a numpy array (float32 arrays are "f32")."""
    return {np.dtype(np.float32): "f32", np.dtype(np.float16): "f16"}[np.asarray(x).dtype]


def merge_types(a, b):
    """Nx type promotion between two float types (f16 and bf16 merge to f32)."""
    if a == b:
        return a
    return "f32"


def nbits_sizes(attrs):
    """``quantized.ex:226-228``: K, N, bits (default 4) and block_size. ``accuracy_level`` is
    never read by the reference, so it changes nothing here either."""
    return int(attrs["K"]), int(attrs["N"]), int(attrs.get("bits", 4)), int(attrs["block_size"])


def unpack(packed, bits):
    """``packed.ex:9-23``: the ``bits``-wide unsigned values of each byte on the last axis,
    lowest bits first (element 2i of a 4-bit tensor is the low nibble of byte i), as s16.
    8-bit values are returned unchanged."""
    packed = np.asarray(packed)
    if bits == 8:
        return packed
    per = 8 // bits
    shifts = np.arange(per, dtype=np.int16) * bits
    values = (packed.astype(np.int16) & 255)[..., None] >> shifts
    values = values & (2 ** bits - 1)
    return values.reshape(*packed.shape[:-1], packed.shape[-1] * per)


def unpack_signed(packed, bits):
    """``quantized.ex:294-300``: sign extension of s8-typed packed data. MatMulNBits' B is u8
    (``transmuter.ex:1222-1225``), so on this operator it is the plain ``unpack``."""
    values = unpack(packed, bits)
    if bits < 8 and np.asarray(packed).dtype == np.int8:
        values = values - (values >= 2 ** (bits - 1)) * 2 ** bits
    return values


def block_zero_points(zero, shape, bits, t, signed=False):
    """``quantized.ex:306-325``: the zero point of each block. None -> 2^(bits-1) (0 for signed
    data); a float tensor -> reshaped to ``shape`` and cast to ``t``; packed integers ->
    reshaped to rows, unpacked, sliced to the block count, cast to ``t``."""
    if zero is None:
        return as_type(0 if signed else 2 ** (bits - 1), t)
    zero = np.asarray(zero)
    if zero.dtype.kind == "f":
        return as_type(zero.reshape(shape), t)
    rows = zero.reshape(*shape[:-1], -1)
    blocks = shape[-1]
    return as_type(unpack_signed(rows, bits)[..., :blocks], t)


def _sub(a, b, t):
    """Subtraction in float type ``t`` with one rounding."""
    if t == "f32":
        return (np.asarray(a, np.float32) - np.asarray(b, np.float32)).astype(np.float32)
    if t == "f16":
        return (np.asarray(a, np.float64) - np.asarray(b, np.float64)).astype(np.float16)
    return round_bf16_from_f64(np.asarray(a, np.float64) - np.asarray(b, np.float64))


def _mul(a, b, t):
    """Multiplication in float type ``t`` with one rounding (products of two f16 or two bf16
    values are exact in float64, so rounding that product once is the typed multiply)."""
    if t == "f32":
        return (np.asarray(a, np.float32) * np.asarray(b, np.float32)).astype(np.float32)
    if t == "f16":
        return (np.asarray(a, np.float64) * np.asarray(b, np.float64)).astype(np.float16)
    return round_bf16_from_f64(np.asarray(a, np.float64) * np.asarray(b, np.float64))


def dequantize(q, zero, scales, t):
    """``packed.ex:28-36``: ``(q - zero) * scales`` per block of the last axis of q, each step
    in type ``t``."""
    blocks = scales.shape
    qb = q.reshape(*blocks, -1)
    z = np.asarray(zero)
    z = z[..., None] if z.ndim else z
    d = _mul(_sub(qb, z, t), np.asarray(scales)[..., None], t)
    return d.reshape(q.shape)


def dequantize_weight(b, scales, zero_points, k, n, bits, block_size, t):
    """``quantized.ex:234-240``: the {N, K} weights in float type ``t``: B unpacked and
    reshaped to {N, blocks*block_size}, the scales and zero points per block, the dequantize,
    then the slice to K columns."""
    blocks = -(-k // block_size)
    q = as_type(unpack_signed(np.asarray(b).reshape(n, -1), bits).reshape(n, blocks * block_size), t)
    s = as_type(np.asarray(scales).reshape(n, blocks), t)
    z = block_zero_points(zero_points, (n, blocks), bits, t)
    return dequantize(q, z, s, t)[:, :k]


def upcast(x, compute_type):
    """``transmuter.ex:1323-1327``: f16/bf16 become ``compute_type`` when one is given."""
    if compute_type is None:
        return x
    t = type_of(x) if not isinstance(x, tuple) else x[1]
    return as_type(x, compute_type) if t in ("f16", "bf16") else x


def moved_weight(b, scales, zero_points, attrs, scales_type, compute_type=None):
    """``transmuter.ex:1230-1240``: the weight that ``move/2`` builds once at load, in the
    scales' type after ``compute_type`` (f16/bf16 scales become ``compute_type``)."""
    k, n, bits, bs = nbits_sizes(attrs)
    t = scales_type if (compute_type is None or scales_type == "f32") else compute_type
    return dequantize_weight(b, scales, zero_points, k, n, bits, bs, t), t


def dot(a, w, out_type):
    """``Nx.dot(a, [-1], w, [1])`` (``quantized.ex:44``). The accumulation is done in float64
    (the reference delegates it to XLA; its order is not part of the contract), then the
    result is rounded once to ``out_type``."""
    a64 = np.asarray(a, np.float64)
    w64 = np.asarray(w, np.float64)
    y = a64.reshape(-1, a64.shape[-1]) @ w64.T
    return as_type(y.astype(np.float32) if out_type == "bf16" else y, out_type).reshape(*a64.shape[:-1], w64.shape[0])


def matmul_nbits(attrs, a, b, scales, zero_points=None, g_idx=None, bias=None,
                 a_type=None, bias_type=None):
    """``quantized.ex:30-46``: the MatMulNBits clause for a model without a backend (the weight
    is dequantized in the graph, in A's type).

    ``a_type`` names A's float type when A is carried as float32 holding bf16 values. A B that
    is already an {N, K} weight (a moved model, ``quantized.ex:39-42``) is used as is.
    Returns (Y, Y's type)."""
    if g_idx is not None:
        raise ValueError("MatMulNBits with the g_idx input is not supported")
    k, n, bits, bs = nbits_sizes(attrs)
    t = a_type or type_of(a)
    if np.asarray(b).shape == (n, k):
        w, wt = np.asarray(b), (type_of(b) if np.asarray(b).dtype != np.float32 else "f32")
    else:
        w, wt = dequantize_weight(b, scales, zero_points, k, n, bits, bs, t), t
    out_t = merge_types(t, wt)
    y = dot(a, w, out_t)
    if bias is not None:
        bt = bias_type or type_of(bias)
        out_t = merge_types(out_t, bt)
        y = as_type(np.asarray(y, np.float64) + np.asarray(bias, np.float64), out_t)
    return y, out_t


def gather_block_quantized(attrs, data, indices, scales, zero_points=None):
    """``quantized.ex:49-66``: rows of a table quantized along its last axis, gathered on axis
    0 and dequantized in the scales' type."""
    bits = int(attrs.get("bits", 4))
    if int(attrs.get("gather_axis", 0)) != 0:
        raise ValueError("GatherBlockQuantized supports gather_axis 0 and quantize_axis on the last axis")
    t = type_of(scales)
    q = as_type(unpack_signed(np.take(data, indices, axis=0), bits), t)
    shape = q.shape[:-1] + (scales.shape[-1],)
    zp = None if zero_points is None else np.take(zero_points, indices, axis=0)
    zero = block_zero_points(zp, shape, bits, t, signed=np.asarray(data).dtype == np.int8)
    return dequantize(q, zero, np.take(scales, indices, axis=0), t)


def within_reference_tolerance(actual, expected):
    """``test/transmuter/ops_test.exs:582-598``: max |actual - expected| <= 1e-4 + 1e-3 *
    max |expected| over the finite expected values."""
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    diff = np.abs(actual - expected)
    diff[np.isnan(expected) & np.isnan(actual)] = 0
    diff[actual == expected] = 0
    finite = np.isfinite(expected)
    tol = 1e-4 + 1e-3 * (np.abs(expected[finite]).max() if finite.any() else 0.0)
    return float(diff.max()) if diff.size else 0.0, tol


def rel_l2(actual, expected):
    """||actual - expected||_2 / ||expected||_2 in float64."""
    actual = np.asarray(actual, np.float64).ravel()
    expected = np.asarray(expected, np.float64).ravel()
    den = np.linalg.norm(expected)
    return float(np.linalg.norm(actual - expected) / (den if den > 0 else 1.0))
