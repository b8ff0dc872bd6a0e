"""A q4 decoder (Qwen3-0.6B architecture, random-init weights) whose projections all run through
libtq4's MatMulNBits, for the decode-throughput configuration of the north star.

Every projection is a 4-bit MatMulNBits weight with block 32 and f32 scales ~ U(0.005, 0.02)
and no zero points. The embedding is the GatherBlockQuantized of the tied lm_head weight
(lib/transmuter/emlx.ex:50-53 describes the tied q4 exports). The operators around the projections
follow lib/transmuter/ops/transformer.ex: RMSNorm (:1056-1069), Qwen3's per-head QK-norm,
rotate-half RoPE with theta 1e6 (:558-590), GroupQueryAttention with 16 query / 8 KV heads over an
f32 cache (:106-175), SwiGLU. q/k/v and gate/up run as one MatMulNBits each, merged along N (the
packed form of the sibling merge in lib/transmuter/fusion.ex:430-540): weights given as separate
q, k, v, gate and up inputs, as an ONNX export stores them (``split_siblings``), are merged at load
by ``tq4_weight_merge``.

A step reads its position and token from device memory; one CUDA graph of a step, replayed,
runs prompt prefill (forced tokens) and greedy decoding without the host. A layer is five
launches: the q/k/v projection with the RMSNorm in its activation staging, attention with the
QK-norm and RoPE folded in, the o projection adding into the residual stream in place, the
gate/up projection with the RMSNorm in its staging, and the down projection with SwiGLU in its
staging, adding into the residual stream (tq4_matmul_fused, tq4_attention_decode_rope).
"""

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .quantized import PackedWeight, _ptr


@dataclass(frozen=True)
class DecoderConfig:
    layers: int = 28
    hidden: int = 1024
    inter: int = 3072
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 151936
    eps: float = 1e-6
    theta: float = 1e6
    block_size: int = 32
    max_len: int = 257


QWEN3_0_6B = DecoderConfig()


def rope_tables(cfg):
    """cos/sin [max_len][head_dim/2] in f32 (computed in float64, as an export's caches)."""
    half = cfg.head_dim // 2
    inv = cfg.theta ** (-np.arange(half, dtype=np.float64) * 2.0 / cfg.head_dim)
    ang = np.arange(cfg.max_len, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def random_weights(cfg, seed=0):
    """Seeded q4 weights: uniform bytes (two uniform nibbles each), f32 scales ~ U(0.005, 0.02).
    Returns {name: (B [N, blocks, bs/2] u8, scales [N*blocks] f32)} with q/k/v and gate/up merged."""
    r = np.random.default_rng(seed)
    bs = cfg.block_size

    def q4(n, k):
        blocks = -(-k // bs)
        b = r.integers(0, 256, (n, blocks, bs // 2), dtype=np.uint8)
        s = (r.random(n * blocks, dtype=np.float32) * 0.015 + 0.005).astype(np.float32)
        return b, s

    w = {}
    qkv_n = (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim
    for layer in range(cfg.layers):
        w[f"{layer}.qkv"] = q4(qkv_n, cfg.hidden)
        w[f"{layer}.o"] = q4(cfg.hidden, cfg.heads * cfg.head_dim)
        w[f"{layer}.gate_up"] = q4(2 * cfg.inter, cfg.hidden)
        w[f"{layer}.down"] = q4(cfg.hidden, cfg.inter)
    w["lm_head"] = q4(cfg.vocab, cfg.hidden)
    return w


# The sibling projections that read one input, merged along N (the packed form of
# Fusion.matmuls/2, lib/transmuter/fusion.ex:430-540).
SIBLINGS = {"qkv": ("q", "k", "v"), "gate_up": ("gate", "up")}


def sibling_sizes(cfg):
    return {"qkv": [cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim],
            "gate_up": [cfg.inter, cfg.inter]}


def split_siblings(weights, cfg):
    """The weights as a q4 ONNX export stores them: one MatMulNBits input each for q, k, v, gate
    and up (the row ranges of the merged projections of ``random_weights``)."""
    sizes = sibling_sizes(cfg)
    out = {}
    for name, (b, s) in weights.items():
        layer, _, proj = name.rpartition(".")
        if proj not in SIBLINGS:
            out[name] = (b, s)
            continue
        blocks, r0 = b.shape[1], 0
        for part, n in zip(SIBLINGS[proj], sizes[proj]):
            out[f"{layer}.{part}"] = (b[r0:r0 + n], s[r0 * blocks:(r0 + n) * blocks])
            r0 += n
    return out


class Q4Decoder:
    """The decoder on one GPU. Norm weights are 1 (the configuration's choice)."""

    def __init__(self, cfg=QWEN3_0_6B, seed=0, device="cuda:0", weights=None):
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        host = weights if weights is not None else random_weights(cfg, seed)
        self.weights = {}
        for name, (b, s) in host.items():
            n = b.shape[0]
            k = cfg.inter if name.endswith(".down") else (cfg.heads * cfg.head_dim if name.endswith(".o") else cfg.hidden)
            self.weights[name] = PackedWeight((k, n, 4, cfg.block_size), torch.from_numpy(b).to(dev),
                                              torch.from_numpy(s).to(dev), None, dtype=torch.float32, device=dev)
        # Separate sibling inputs (an ONNX export's q, k, v and gate, up) merge into one handle
        # each, so one GEMV streams the whole group's rows.
        for layer in range(cfg.layers):
            for merged, parts in SIBLINGS.items():
                names = [f"{layer}.{p}" for p in parts]
                if all(n in self.weights for n in names):
                    ws = [self.weights.pop(n) for n in names]
                    self.weights[f"{layer}.{merged}"] = PackedWeight.merge(ws)
                    for w in ws:
                        w.close()
        f32 = dict(dtype=torch.float32, device=dev)
        self.ones_h = torch.ones(cfg.hidden, **f32)
        self.ones_d = torch.ones(cfg.head_dim, **f32)
        cos, sin = rope_tables(cfg)
        self.cos, self.sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
        kv = (cfg.layers, cfg.kv_heads, cfg.max_len, cfg.head_dim)
        self.k_cache, self.v_cache = torch.zeros(kv, **f32), torch.zeros(kv, **f32)
        qkv_n = (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim
        self.x = torch.zeros(cfg.hidden, **f32)        # residual stream
        self.qkv = torch.zeros(qkv_n, **f32)
        self.attn = torch.zeros(cfg.heads * cfg.head_dim, **f32)
        self.gu = torch.zeros(2 * cfg.inter, **f32)
        self.logits = torch.zeros(cfg.vocab, **f32)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.forced = torch.full((cfg.max_len,), -1, dtype=torch.int64, device=dev)  # -1: greedy
        self.log = torch.zeros(cfg.max_len, dtype=torch.int64, device=dev)
        self.graph = None
        self._lib = _lib.load()
        self._bind()

    def _bind(self):
        lib = self._lib
        vp, i64, i32, f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        sigs = {
            "tq4_add_rmsnorm": [vp, vp, vp, vp, i64, i64, f, vp],
            "tq4_qk_norm_rope": [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f, vp],
            "tq4_attention_decode": [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp],
            "tq4_silu_mul": [vp, vp, vp, i64, vp],
            "tq4_argmax_advance": [vp, i64, vp, i32, vp, vp, vp, i32, vp],
            "tq4_attention_decode_rope": [vp, vp, vp, vp, vp, vp, vp, f, vp, vp, vp, vp, i32, i32, i32, i32, vp],
            "tq4_matmul_fused": [vp, vp, vp, vp, f, i32, vp, vp, vp],
        }
        for name, args in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def step(self):
        """One token: embedding of *token at *pos through every layer, then the greedy step."""
        cfg, lib, st, chk = self.cfg, self._lib, self._stream(), _lib.check
        p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
        qd = cfg.heads * cfg.head_dim
        kd = cfg.kv_heads * cfg.head_dim
        lm = self.weights["lm_head"]
        chk(lib.tq4_gather_rows(lm._handle, p(self.token), 1, p(self.x), st))  # tied embedding
        for layer in range(cfg.layers):
            w = lambda name: self.weights[f"{layer}.{name}"]._handle
            chk(lib.tq4_matmul_fused(w("qkv"), p(self.x), None, p(self.ones_h), cfg.eps, 1, None, p(self.qkv), st))
            q, k, v = self.qkv[:qd], self.qkv[qd:qd + kd], self.qkv[qd + kd:]
            chk(lib.tq4_attention_decode_rope(p(q), p(k), p(v), p(self.ones_d), p(self.ones_d), p(self.cos),
                                              p(self.sin), cfg.eps, p(self.k_cache[layer]), p(self.v_cache[layer]),
                                              p(self.pos), p(self.attn), cfg.heads, cfg.kv_heads, cfg.head_dim,
                                              cfg.max_len, st))
            chk(lib.tq4_matmul_fused(w("o"), p(self.attn), None, None, 0.0, 0, p(self.x), p(self.x), st))
            chk(lib.tq4_matmul_fused(w("gate_up"), p(self.x), None, p(self.ones_h), cfg.eps, 1, None, p(self.gu), st))
            chk(lib.tq4_matmul_fused(w("down"), p(self.gu[:cfg.inter]), p(self.gu[cfg.inter:]), None, 0.0, 2,
                                     p(self.x), p(self.x), st))
        chk(lib.tq4_matmul_fused(lm._handle, p(self.x), None, p(self.ones_h), cfg.eps, 1, None, p(self.logits), st))
        chk(lib.tq4_argmax_advance(p(self.logits), cfg.vocab, p(self.forced), cfg.max_len, p(self.pos),
                                   p(self.token), p(self.log), cfg.max_len, st))

    LAUNCHES_PER_LAYER = 5
    LAUNCHES_PER_STEP_EXTRA = 3  # embedding gather, lm_head, argmax

    def reset(self, prompt):
        """Starts a sequence: the prompt's tokens are forced, position 0 holds prompt[0]."""
        prompt = torch.as_tensor(prompt, dtype=torch.int64)
        n = prompt.numel()
        assert 0 < n < self.cfg.max_len
        self.forced.fill_(-1)
        self.forced[:n] = prompt.to(self.device)
        self.pos.zero_()
        self.token.copy_(prompt[:1].to(self.device))
        self.log.zero_()
        self.log[:1] = prompt[:1].to(self.device)
        self.k_cache.zero_()
        self.v_cache.zero_()

    def capture(self):
        """Captures one step as a CUDA graph (after one eager step to create workspaces)."""
        s = torch.cuda.Stream(self.device)
        with torch.cuda.stream(s):
            saved = (self.pos.clone(), self.token.clone(), self.log.clone())
            self.step()
            torch.cuda.synchronize(self.device)
            self.pos.copy_(saved[0])
            self.token.copy_(saved[1])
            self.log.copy_(saved[2])
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self.step()
        torch.cuda.synchronize(self.device)

    def run(self, steps):
        """`steps` graph replays (or eager steps before capture)."""
        for _ in range(steps):
            if self.graph is not None:
                self.graph.replay()
            else:
                self.step()

    def generate(self, prompt, new_tokens):
        """Prefill the prompt (forced steps) then `new_tokens` greedy tokens; returns them."""
        self.reset(prompt)
        n = len(prompt)
        self.run(n - 1 + new_tokens)
        torch.cuda.synchronize(self.device)
        return self.log[n:n + new_tokens].cpu().numpy()
