"""CPU oracle of the q4 decoder (TEST INFRASTRUCTURE ONLY: tests and bench's CPU baseline use it).

A numpy restatement, in float64, of the operators the decode configuration chains around
MatMulNBits, following georgeguimaraes/transmuter 2.0.0 lib/transmuter/ops/transformer.ex:
- rms_norm/4 (:1056-1069): x * rsqrt(mean(x^2) + eps) * w, and the residual add of
  SkipSimplifiedLayerNormalization (:297-300);
- rotate/4 (:558-590), interleaved = 0: [x1 cos - x2 sin, x2 cos + x1 sin] on the two halves;
- GroupQueryAttention (:106-175) for one query row: causal over the cache, scale 1/sqrt(head_dim)
  (:1089-1094), query head h reads KV head h // (heads / kv_heads);
- SwiGLU silu(gate) * up; greedy argmax (lowest index among equal maxima).
The projections use oracle.matmul_nbits.dequantize_weight (quantized.ex:234-240), in f32.
Parity of this file rests on matmul_nbits (pinned to the reference fixtures) and on these
textbook operator definitions; the decoder graph itself has no reference fixture.
"""

import numpy as np

from . import matmul_nbits as o


def rms_norm(x, w, eps):
    x = np.asarray(x)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def rope(x, cos, sin):
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1)


class OracleDecoder:
    """dtype float64 (default) is the parity oracle; float32 is the moved-weight CPU path that the
    benchmark times (dense f32 weights, BLAS matrix-vector products, as EXLA's CPU client runs a
    moved model)."""

    def __init__(self, cfg, weights, cos, sin, dtype=np.float64):
        self.cfg = cfg
        self.dt = dtype
        self.cos, self.sin = np.asarray(cos, dtype), np.asarray(sin, dtype)
        self.w = {}
        for name, (b, s) in weights.items():
            n = b.shape[0]
            k = cfg.inter if name.endswith(".down") else (cfg.heads * cfg.head_dim if name.endswith(".o") else cfg.hidden)
            self.w[name] = o.dequantize_weight(b, s, None, k, n, 4, cfg.block_size, "f32").astype(dtype)
        self.k_cache = np.zeros((cfg.layers, cfg.kv_heads, cfg.max_len, cfg.head_dim), dtype)
        self.v_cache = np.zeros_like(self.k_cache)

    def step(self, token, pos):
        """Logits of `token` at position `pos` (updates the cache)."""
        c = self.cfg
        qd, kd = c.heads * c.head_dim, c.kv_heads * c.head_dim
        x = self.w["lm_head"][token].copy()  # tied embedding
        g = c.heads // c.kv_heads
        for layer in range(c.layers):
            h = rms_norm(x, 1.0, c.eps)
            qkv = self.w[f"{layer}.qkv"] @ h
            q = qkv[:qd].reshape(c.heads, c.head_dim)
            k = qkv[qd:qd + kd].reshape(c.kv_heads, c.head_dim)
            v = qkv[qd + kd:].reshape(c.kv_heads, c.head_dim)
            q = rope(rms_norm(q, 1.0, c.eps), self.cos[pos], self.sin[pos])
            k = rope(rms_norm(k, 1.0, c.eps), self.cos[pos], self.sin[pos])
            self.k_cache[layer, :, pos] = k
            self.v_cache[layer, :, pos] = v
            out = np.zeros((c.heads, c.head_dim), self.dt)
            for hh in range(c.heads):
                kc = self.k_cache[layer, hh // g, :pos + 1]
                vc = self.v_cache[layer, hh // g, :pos + 1]
                s = kc @ q[hh] / np.sqrt(c.head_dim)
                p = np.exp(s - s.max())
                out[hh] = (p / p.sum()) @ vc
            x = x + self.w[f"{layer}.o"] @ out.reshape(-1)
            h = rms_norm(x, 1.0, c.eps)
            gu = self.w[f"{layer}.gate_up"] @ h
            gate, up = gu[:c.inter], gu[c.inter:]
            x = x + self.w[f"{layer}.down"] @ (gate / (1 + np.exp(-gate)) * up)
        return self.w["lm_head"] @ rms_norm(x, 1.0, c.eps)

    def generate(self, prompt, new_tokens):
        """Forced prompt then greedy tokens; returns (generated tokens, logits of every step)."""
        logits, out = [], []
        tok = int(prompt[0])
        for pos in range(len(prompt) - 1 + new_tokens):
            lg = self.step(tok, pos)
            logits.append(lg)
            nxt = int(prompt[pos + 1]) if pos + 1 < len(prompt) else int(np.argmax(lg))
            if pos + 1 >= len(prompt):
                out.append(nxt)
            tok = nxt
        return np.array(out), np.array(logits)
