"""The decoder oracle (oracle/decoder.py) checked against an independent statement of the same
network: one causal forward over the whole sequence in torch float64 (scaled_dot_product_attention
with grouped KV heads), which must give the oracle's incremental, cache-based logits at every
position. CPU only, tiny configuration."""

import numpy as np
import torch
import torch.nn.functional as F

from oracle import matmul_nbits as o
from oracle.decoder import OracleDecoder
from transmuter_b200.decoder import DecoderConfig, random_weights, rope_tables

TINY = DecoderConfig(layers=2, hidden=256, inter=512, heads=4, kv_heads=2, head_dim=64, vocab=1000, max_len=40)


def dense(cfg, weights):
    out = {}
    for name, (b, s) in weights.items():
        k = cfg.inter if name.endswith(".down") else (cfg.heads * cfg.head_dim if name.endswith(".o") else cfg.hidden)
        out[name] = torch.from_numpy(o.dequantize_weight(b, s, None, k, b.shape[0], 4, cfg.block_size, "f32").astype(np.float64))
    return out


def full_forward(cfg, w, cos, sin, tokens):
    def rms(x):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + cfg.eps)

    def rope(x, c, s):  # x [T, heads, D]
        half = x.shape[-1] // 2
        x1, x2 = x[..., :half], x[..., half:]
        c, s = c[:, None, :], s[:, None, :]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)

    t = len(tokens)
    qd, kd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    c = torch.from_numpy(cos[:t].astype(np.float64))
    s = torch.from_numpy(sin[:t].astype(np.float64))
    x = w["lm_head"][torch.as_tensor(tokens)]
    for layer in range(cfg.layers):
        qkv = rms(x) @ w[f"{layer}.qkv"].T
        q = rope(rms(qkv[:, :qd].view(t, cfg.heads, cfg.head_dim)), c, s)
        k = rope(rms(qkv[:, qd:qd + kd].view(t, cfg.kv_heads, cfg.head_dim)), c, s)
        v = qkv[:, qd + kd:].view(t, cfg.kv_heads, cfg.head_dim)
        att = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                             is_causal=True, enable_gqa=True)
        x = x + att.transpose(0, 1).reshape(t, qd) @ w[f"{layer}.o"].T
        gu = rms(x) @ w[f"{layer}.gate_up"].T
        gate, up = gu[:, :cfg.inter], gu[:, cfg.inter:]
        x = x + (F.silu(gate) * up) @ w[f"{layer}.down"].T
    return (rms(x) @ w["lm_head"].T).numpy()


def test_incremental_oracle_matches_full_causal_forward():
    weights = random_weights(TINY, seed=3)
    cos, sin = rope_tables(TINY)
    prompt = np.random.default_rng(4).integers(0, TINY.vocab, 6)
    tokens, logits = OracleDecoder(TINY, weights, cos, sin).generate(prompt, 5)
    seq = np.concatenate([prompt, tokens[:-1]])
    full = full_forward(TINY, dense(TINY, weights), cos, sin, seq)
    assert full.shape == logits.shape
    assert o.rel_l2(logits, full) < 1e-12
    assert int(np.argmax(full[-1])) == int(tokens[-1])
    # greedy tokens are the argmax of the logits one position earlier
    assert np.array_equal(np.argmax(full[len(prompt) - 1:], axis=1), tokens)


def test_rope_tables_identity_at_position_zero():
    cos, sin = rope_tables(TINY)
    assert np.all(cos[0] == 1) and np.all(sin[0] == 0)
    assert cos.shape == (TINY.max_len, TINY.head_dim // 2)


def test_split_siblings_are_row_ranges_of_the_merged_projections():
    """split_siblings gives the separate q/k/v and gate/up inputs of an ONNX export; their rows
    concatenated are the merged projections (what tq4_weight_merge builds on the GPU)."""
    from transmuter_b200.decoder import SIBLINGS, sibling_sizes, split_siblings
    weights = random_weights(TINY, seed=5)
    parts = split_siblings(weights, TINY)
    sizes = sibling_sizes(TINY)
    for layer in range(TINY.layers):
        for merged, names in SIBLINGS.items():
            b, s = weights[f"{layer}.{merged}"]
            pb = [parts[f"{layer}.{n}"][0] for n in names]
            ps = [parts[f"{layer}.{n}"][1] for n in names]
            assert [x.shape[0] for x in pb] == sizes[merged]
            assert np.array_equal(np.concatenate(pb), b) and np.array_equal(np.concatenate(ps), s)
            assert f"{layer}.{merged}" not in parts
    assert parts["lm_head"][0] is weights["lm_head"][0]
