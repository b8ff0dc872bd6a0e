"""Seeded synthetic MatMulNBits problems with the shapes and value distributions of the north-star
configs (no model weights, datasets or prompts are used or needed).

Seeds follow the reference fixture generator's convention: crc32 of the case name
(test/support/make_op_fixtures.py:33-35). Nibbles are uniform over [0, 2^bits) and packed lowest
bits first (packed.ex:3), A ~ N(0, 1), scales ~ U(lo, hi).
"""

import zlib
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Config:
    name: str
    k: int
    n: int
    m: int
    bits: int = 4
    block_size: int = 32
    scale_type: str = "f32"
    scale_range: tuple = (0.005, 0.02)
    zp: str = "none"           # none | packed | float
    a_type: str = "f32"
    bias: bool = False
    metric: str = "GB/s"       # GB/s (HBM-bound) or TFLOP/s (tensor-bound)

    @property
    def blocks(self):
        return -(-self.k // self.block_size)

    def weight_bytes(self):
        """Algorithmic bytes of B, scales and zero points as the operator receives them."""
        b = self.n * self.blocks * self.block_size * self.bits // 8
        s = self.n * self.blocks * (4 if self.scale_type == "f32" else 2)
        z = 0
        if self.zp == "packed":
            z = self.n * -(-self.blocks * self.bits // 8)
        elif self.zp == "float":
            z = s
        return b + s + z

    def io_bytes(self):
        asz = 4 if self.a_type == "f32" else 2
        return self.m * self.k * asz + self.m * self.n * asz

    def algorithmic_bytes(self):
        return self.weight_bytes() + self.io_bytes()

    def flops(self):
        return 2 * self.m * self.n * self.k


# The north-star configs (C1..C5). C4 (the decoder) is not a single operator call.
CONFIGS = {
    "c1": Config("c1-decode-1x1024x3072", 1024, 3072, 1, metric="GB/s"),
    "c2": Config("c2-prefill-512x1024x3072", 1024, 3072, 512, scale_type="f16", zp="packed",
                 a_type="f16", metric="TFLOP/s"),
    "c3m1": Config("c3-lmhead-1x1024x151936", 1024, 151936, 1, metric="GB/s"),
    "c3m64": Config("c3-lmhead-64x1024x151936", 1024, 151936, 64, metric="GB/s"),
}
for _m in (1, 16, 256, 4096):
    for _k, _n in ((4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)):
        CONFIGS[f"c5-{_k}x{_n}-m{_m}"] = Config(
            f"c5-llama-{_m}x{_k}x{_n}", _k, _n, _m, block_size=128, scale_type="f16",
            scale_range=(0.002, 0.01), zp="packed", a_type="f16",
            metric="GB/s" if _m <= 16 else "TFLOP/s")


def rng_for(name):
    return np.random.default_rng(zlib.crc32(name.encode()))


def pack(q, bits):
    """Packs unsigned values < 2^bits along the last axis, lowest bits first."""
    per = 8 // bits
    q = np.asarray(q).reshape(*np.shape(q)[:-1], -1, per).astype(np.uint8)
    out = np.zeros(q.shape[:-1], np.uint8)
    for i in range(per):
        out |= (q[..., i] << (bits * i)).astype(np.uint8)
    return out


def _bf16(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)).view(np.float32)


def _float(x, t):
    x = np.asarray(x, np.float32)
    if t == "f16":
        return x.astype(np.float16)
    if t == "bf16":
        return _bf16(x)  # carried as float32 holding bf16 values
    return x


def make(cfg, m=None, seed_name=None):
    """Inputs of one problem: dict with B [N, blocks, bs*bits/8] u8, scales [N*blocks], zp
    (packed u8 [N*ceil(blocks*bits/8)] or float [N*blocks] or None), A [M, K], bias or None."""
    r = rng_for(seed_name or cfg.name)
    m = cfg.m if m is None else m
    blocks = cfg.blocks
    q = r.integers(0, 2 ** cfg.bits, (cfg.n, blocks * cfg.block_size), dtype=np.uint8)
    b = pack(q, cfg.bits).reshape(cfg.n, blocks, cfg.block_size * cfg.bits // 8)
    lo, hi = cfg.scale_range
    scales = _float(r.random(cfg.n * blocks, dtype=np.float32) * (hi - lo) + lo, cfg.scale_type)
    zp = None
    if cfg.zp == "packed":
        zq = r.integers(0, 2 ** cfg.bits, (cfg.n, -(-blocks * cfg.bits // 8) * 8 // cfg.bits), dtype=np.uint8)
        zp = pack(zq, cfg.bits).reshape(-1)
    elif cfg.zp == "float":
        zp = _float(r.random(cfg.n * blocks, dtype=np.float32) * 2 ** cfg.bits, cfg.scale_type)
    a = _float(r.standard_normal((m, cfg.k), dtype=np.float32), cfg.a_type)
    bias = _float(r.standard_normal(cfg.n, dtype=np.float32), cfg.a_type) if cfg.bias else None
    return {"B": b, "scales": scales, "zp": zp, "A": a, "bias": bias,
            "attrs": {"K": cfg.k, "N": cfg.n, "bits": cfg.bits, "block_size": cfg.block_size}}
