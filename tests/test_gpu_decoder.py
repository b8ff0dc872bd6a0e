"""GPU tests of the q4 decoder (transmuter_b200.decoder): every projection through libtq4's
MatMulNBits, the surrounding kernels of include/tq4_decoder.h, graph replay.

- tiny configuration against the float64 oracle (oracle/decoder.py): logits of every step within
  rel-L2 1e-3 (f32 activations), greedy tokens equal;
- graph replay against eager steps: identical tokens and logits (the kernels are deterministic);
- the full Qwen3-0.6B shape against a torch fp32 restatement over the bit-exact dequantized
  weights (tq4_dequantize): logits of the first steps within rel-L2 1e-3;
- positions past the cache set the device status and write nothing.
"""

import ctypes

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import matmul_nbits as o
from oracle.decoder import OracleDecoder
from transmuter_b200 import _lib
from transmuter_b200.decoder import QWEN3_0_6B, DecoderConfig, Q4Decoder, random_weights, rope_tables, split_siblings

pytestmark = pytest.mark.gpu

TINY = DecoderConfig(layers=2, hidden=256, inter=512, heads=4, kv_heads=2, head_dim=64, vocab=1000, max_len=40)
LOGIT_TOL = 1e-3  # rel-L2, f32 activations


def step_logits(dec, prompt, new_tokens):
    dec.reset(prompt)
    out = []
    for _ in range(len(prompt) - 1 + new_tokens):
        dec.run(1)
        out.append(dec.logits.cpu().numpy().astype(np.float64))
    torch.cuda.synchronize()
    n = len(prompt)
    return dec.log[n:n + new_tokens].cpu().numpy(), np.array(out)


@pytest.fixture(scope="module")
def tiny():
    weights = random_weights(TINY, seed=11)
    prompt = np.random.default_rng(12).integers(0, TINY.vocab, 8)
    cos, sin = rope_tables(TINY)
    ref_tokens, ref_logits = OracleDecoder(TINY, weights, cos, sin).generate(prompt, 8)
    return weights, prompt, ref_tokens, ref_logits


def test_tiny_decoder_matches_oracle(tiny):
    weights, prompt, ref_tokens, ref_logits = tiny
    dec = Q4Decoder(TINY, weights=weights)
    tokens, logits = step_logits(dec, prompt, 8)
    for i in range(len(logits)):
        assert o.rel_l2(logits[i], ref_logits[i]) < LOGIT_TOL, i
    assert np.array_equal(tokens, ref_tokens)


def test_separate_sibling_inputs_merge_into_the_same_decoder(tiny):
    """q, k, v and gate, up given as separate MatMulNBits inputs (an ONNX export) are merged at
    load by tq4_weight_merge: the merged handles equal the pre-merged ones bit for bit, so the
    logits and tokens are identical."""
    weights, prompt, ref_tokens, _ = tiny
    merged = Q4Decoder(TINY, weights=weights)
    separate = Q4Decoder(TINY, weights=split_siblings(weights, TINY))
    assert sorted(separate.weights) == sorted(merged.weights)
    for name in merged.weights:
        assert torch.equal(separate.weights[name].dequantize(), merged.weights[name].dequantize()), name
    want_tokens, want_logits = step_logits(merged, prompt, 8)
    got_tokens, got_logits = step_logits(separate, prompt, 8)
    assert np.array_equal(got_tokens, want_tokens) and np.array_equal(got_tokens, ref_tokens)
    assert np.array_equal(got_logits, want_logits)


def test_tiny_graph_replay_matches_eager(tiny):
    weights, prompt, ref_tokens, _ = tiny
    dec = Q4Decoder(TINY, weights=weights)
    eager_tokens, eager_logits = step_logits(dec, prompt, 8)
    dec.capture()
    graph_tokens, graph_logits = step_logits(dec, prompt, 8)
    assert np.array_equal(graph_tokens, eager_tokens)
    assert np.array_equal(graph_logits, eager_logits)
    assert np.array_equal(dec.generate(prompt, 8), ref_tokens)


def test_position_past_cache_sets_device_status(tiny):
    weights = tiny[0]
    dec = Q4Decoder(TINY, weights=weights)
    lib = dec._lib
    code = ctypes.c_int32(0)
    _lib.check(lib.tq4_device_status(0, ctypes.byref(code)))
    dec.reset([1, 2])
    dec.pos.fill_(TINY.max_len)  # one past the last cache row
    k_before = dec.k_cache.clone()
    dec.run(1)
    _lib.check(lib.tq4_device_status(0, ctypes.byref(code)))
    assert code.value == 0x200
    assert torch.equal(dec.k_cache, k_before)


@pytest.mark.parametrize("pos", [0, 1, 31, 32, 33, 100, 255, 256])
@pytest.mark.parametrize("heads,kv_heads,head_dim", [(16, 8, 128), (8, 2, 64), (4, 4, 256)])
def test_attention_decode_against_torch(pos, heads, kv_heads, head_dim):
    """tq4_attention_decode over positions that end inside, on and past 32-position chunks (the
    chunk-combine path) against an fp64 softmax over the same cache; the new row lands in the cache."""
    lib = _lib.load()
    max_len = 257
    g = torch.Generator().manual_seed(pos * 7 + heads)
    dev = torch.device("cuda:0")
    q = torch.randn(heads, head_dim, generator=g)
    k_new = torch.randn(kv_heads, head_dim, generator=g)
    v_new = torch.randn(kv_heads, head_dim, generator=g)
    k_cache = torch.randn(kv_heads, max_len, head_dim, generator=g)
    v_cache = torch.randn(kv_heads, max_len, head_dim, generator=g)
    k_ref, v_ref = k_cache.double().clone(), v_cache.double().clone()
    k_ref[:, pos], v_ref[:, pos] = k_new.double(), v_new.double()
    grp = heads // kv_heads
    ref = torch.empty(heads, head_dim, dtype=torch.float64)
    for h in range(heads):
        s = k_ref[h // grp, :pos + 1] @ q[h].double() / head_dim ** 0.5
        ref[h] = torch.softmax(s, 0) @ v_ref[h // grp, :pos + 1]
    d = [t.to(dev).contiguous() for t in (q, k_new, v_new, k_cache, v_cache)]
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    out = torch.empty(heads, head_dim, device=dev)
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    fn = lib.tq4_attention_decode
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    for _ in range(2):  # twice: a call leaves nothing behind that changes the next
        _lib.check(fn(*[vp(t) for t in d], vp(p), vp(out), heads, kv_heads, head_dim, max_len,
                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()
        assert o.rel_l2(out.double().cpu().numpy(), ref.numpy()) < 1e-5
    assert torch.equal(d[3][:, pos].cpu(), k_new) and torch.equal(d[4][:, pos].cpu(), v_new)


@pytest.mark.parametrize("max_len,pos", [(40, 0), (40, 39), (33, 32), (1000, 517), (1000, 999), (4096, 3000)])
def test_attention_decode_cache_lengths(max_len, pos):
    """Caches of other lengths: a cluster of fewer than 8 ranks (short caches) and ranks that fold
    several 32-position chunks into their running softmax (long caches)."""
    lib = _lib.load()
    heads, kv_heads, hd = 16, 8, 128
    g = torch.Generator().manual_seed(max_len + pos)
    dev = torch.device("cuda:0")
    q = torch.randn(heads, hd, generator=g)
    k_new, v_new = torch.randn(kv_heads, hd, generator=g), torch.randn(kv_heads, hd, generator=g)
    k_cache = torch.randn(kv_heads, max_len, hd, generator=g)
    v_cache = torch.randn(kv_heads, max_len, hd, generator=g)
    k_ref, v_ref = k_cache.double().clone(), v_cache.double().clone()
    k_ref[:, pos], v_ref[:, pos] = k_new.double(), v_new.double()
    grp = heads // kv_heads
    ref = torch.stack([torch.softmax(k_ref[h // grp, :pos + 1] @ q[h].double() / hd ** 0.5, 0) @ v_ref[h // grp, :pos + 1]
                       for h in range(heads)])
    d = [t.to(dev).contiguous() for t in (q, k_new, v_new, k_cache, v_cache)]
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    out = torch.empty(heads, hd, device=dev)
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    fn = lib.tq4_attention_decode
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    _lib.check(fn(*[vp(t) for t in d], vp(p), vp(out), heads, kv_heads, hd, max_len,
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert o.rel_l2(out.double().cpu().numpy(), ref.numpy()) < 1e-5
    assert torch.equal(d[3][:, pos].cpu(), k_new) and torch.equal(d[4][:, pos].cpu(), v_new)
    untouched = [i for i in range(max_len) if i != pos]
    assert torch.equal(d[3][:, untouched].cpu(), k_cache[:, untouched])


def torch_reference_logits(dec, cfg, prompt, steps):
    """fp32 restatement on the GPU over the dequantized weights (bit-exact to the handles')."""
    w = {name: pw.dequantize().float() for name, pw in dec.weights.items()}
    qd, kd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    cos, sin = dec.cos, dec.sin

    def rms(x):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + cfg.eps)

    def rope(x, c, s):
        half = x.shape[-1] // 2
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * c[:, None] - x2 * s[:, None], x2 * c[:, None] + x1 * s[:, None]], -1)

    t = len(prompt) + steps - 1
    tokens = list(prompt)
    logits = []
    for _ in range(steps):  # recompute the whole causal sequence each step (simple, not fast)
        n = len(tokens)
        x = w["lm_head"][torch.as_tensor(tokens, device=dec.device)]
        c, s = cos[:n], sin[:n]
        for layer in range(cfg.layers):
            qkv = rms(x) @ w[f"{layer}.qkv"].T
            q = rope(rms(qkv[:, :qd].view(n, cfg.heads, cfg.head_dim)), c, s)
            k = rope(rms(qkv[:, qd:qd + kd].view(n, cfg.kv_heads, cfg.head_dim)), c, s)
            v = qkv[:, qd + kd:].view(n, cfg.kv_heads, cfg.head_dim)
            att = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                                 is_causal=True, enable_gqa=True)
            x = x + att.transpose(0, 1).reshape(n, qd) @ w[f"{layer}.o"].T
            gu = rms(x) @ w[f"{layer}.gate_up"].T
            x = x + (F.silu(gu[:, :cfg.inter]) * gu[:, cfg.inter:]) @ w[f"{layer}.down"].T
        lg = rms(x[-1:]) @ w["lm_head"].T
        logits.append(lg[0].double().cpu().numpy())
        tokens.append(int(torch.argmax(lg[0])))
    assert len(tokens) == t + 1
    return np.array(logits), np.array(tokens[len(prompt):])


def test_full_size_decoder_matches_torch_fp32():
    cfg = QWEN3_0_6B
    dec = Q4Decoder(cfg, seed=5)
    prompt = np.random.default_rng(6).integers(0, cfg.vocab, 16)
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False  # a true fp32 reference
    try:
        ref_logits, ref_tokens = torch_reference_logits(dec, cfg, prompt, 3)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved
    dec.capture()
    dec.reset(prompt)
    dec.run(len(prompt) - 1)
    got = []
    for _ in range(3):
        dec.run(1)
        got.append(dec.logits.double().cpu().numpy())
    for i in range(3):
        assert o.rel_l2(got[i], ref_logits[i]) < LOGIT_TOL, i
    n = len(prompt)
    assert np.array_equal(dec.log[n:n + 3].cpu().numpy(), ref_tokens)


def _fused(lib):
    fn = lib.tq4_matmul_fused
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_float, ctypes.c_int] + [ctypes.c_void_p] * 3
    return fn


@pytest.mark.parametrize("prologue", [0, 1, 2])
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("k,n", [(1024, 4096), (3072, 1024), (1024, 151936)])
def test_matmul_fused_matches_unfused(prologue, residual, k, n):
    """tq4_matmul_fused against the same steps done separately (torch fp64 over the handle's
    bit-exact dequantized weight): RMSNorm / SwiGLU prologue, residual epilogue in place."""
    lib = _lib.load()
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(k + n + 7 * prologue)
    from transmuter_b200.quantized import PackedWeight
    blocks = k // 32
    b = torch.randint(0, 256, (n, blocks, 16), dtype=torch.uint8, generator=g)
    s = torch.rand(n * blocks, generator=g) * 0.015 + 0.005
    w = PackedWeight((k, n, 4, 32), b.to(dev), s.to(dev), None, dtype=torch.float32, device=dev)
    x = torch.randn(k, generator=g).to(dev)
    x2 = torch.randn(k, generator=g).to(dev)
    nw = (torch.rand(k, generator=g) + 0.5).to(dev)
    y = torch.randn(n, generator=g).to(dev)
    y0 = y.clone()
    vp = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    _lib.check(_fused(lib)(w._handle, vp(x), vp(x2), vp(nw), 1e-6, prologue, vp(y) if residual else None, vp(y),
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    xd = x.double()
    if prologue == 1:
        a = xd * torch.rsqrt((xd * xd).mean() + 1e-6) * nw.double()
    elif prologue == 2:
        a = xd / (1 + torch.exp(-xd)) * x2.double()
    else:
        a = xd
    want = w.dequantize().double() @ a + (y0.double() if residual else 0)
    assert ((y.double() - want).norm() / want.norm()).item() < 1e-3
    w.close()


@pytest.mark.parametrize("pos", [0, 5, 31, 32, 200])
def test_attention_decode_rope_matches_separate_steps(pos):
    """tq4_attention_decode_rope equals tq4_qk_norm_rope followed by tq4_attention_decode, and
    leaves q / k_new unmodified."""
    lib = _lib.load()
    dev = torch.device("cuda:0")
    heads, kv_heads, hd, max_len = 16, 8, 128, 257
    cfg = DecoderConfig(heads=heads, kv_heads=kv_heads, head_dim=hd, max_len=max_len)
    cos, sin = (torch.from_numpy(t).to(dev) for t in rope_tables(cfg))
    g = torch.Generator().manual_seed(pos + 3)
    q = torch.randn(heads, hd, generator=g).to(dev)
    k = torch.randn(kv_heads, hd, generator=g).to(dev)
    v = torch.randn(kv_heads, hd, generator=g).to(dev)
    qw = (torch.rand(hd, generator=g) + 0.5).to(dev)
    kw = (torch.rand(hd, generator=g) + 0.5).to(dev)
    kc = torch.randn(kv_heads, max_len, hd, generator=g).to(dev)
    vc = torch.randn(kv_heads, max_len, hd, generator=g).to(dev)
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    fr = lib.tq4_attention_decode_rope
    fr.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_float] + [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    out1, kc1, vc1 = torch.empty(heads, hd, device=dev), kc.clone(), vc.clone()
    q0, k0 = q.clone(), k.clone()
    torch.cuda.synchronize()  # the caches are complete before the call (its earlier rows load early)
    _lib.check(fr(vp(q), vp(k), vp(v), vp(qw), vp(kw), vp(cos), vp(sin), 1e-6, vp(kc1), vp(vc1), vp(p), vp(out1),
                  heads, kv_heads, hd, max_len, st))
    torch.cuda.synchronize()
    assert torch.equal(q, q0) and torch.equal(k, k0)
    fq = lib.tq4_qk_norm_rope
    fq.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_void_p]
    fa = lib.tq4_attention_decode
    fa.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    q2, k2, out2, kc2, vc2 = q.clone(), k.clone(), torch.empty(heads, hd, device=dev), kc.clone(), vc.clone()
    _lib.check(fq(vp(q2), vp(k2), vp(qw), vp(kw), vp(cos), vp(sin), vp(p), max_len, heads, kv_heads, hd, 1e-6, st))
    _lib.check(fa(vp(q2), vp(k2), vp(v), vp(kc2), vp(vc2), vp(p), vp(out2), heads, kv_heads, hd, max_len, st))
    torch.cuda.synchronize()
    assert o.rel_l2(out1.double().cpu().numpy(), out2.double().cpu().numpy()) < 1e-5
    assert o.rel_l2(kc1[:, pos].double().cpu().numpy(), kc2[:, pos].double().cpu().numpy()) < 1e-6
    assert torch.equal(vc1, vc2)


@pytest.mark.parametrize("n,offset,kind", [(151936, 0, "ties"), (151937, 1, "nan"), (1000, 3, "ties"),
                                           (7, 0, "neg_inf"), (152000, 2, "plain")])
def test_argmax_advance_rule(n, offset, kind):
    """tq4_argmax_advance: greedy next token = the lowest index among equal maxima, NaN never wins
    (all -inf gives index 0), a forced token wins over the argmax; the log and position advance.
    Ties across the scanning CTAs' slices, odd n and unaligned logits pointers included."""
    lib = _lib.load()
    dev = torch.device("cuda:0")
    r = np.random.default_rng(n + offset)
    x = r.standard_normal(n + offset).astype(np.float32)
    v = x[offset:]
    if kind == "ties":
        top = np.float32(9.0)
        for i in (n - 1, n // 3, n // 2 + 1, 5):
            v[i] = top
    elif kind == "nan":
        v[r.integers(0, n, 50)] = np.nan
        v[n - 2] = np.float32(7.5)
    elif kind == "neg_inf":
        v[:] = -np.inf
    # first occurrence of the maximum = the lowest index among equal maxima; NaN never wins, and
    # an all -inf row gives index 0 (the kernel's rule)
    want = int(np.argmax(np.where(np.isnan(v), -np.inf, v)))
    buf = torch.from_numpy(x).to(dev)
    logits = buf[offset:]
    max_len = 16
    forced = torch.full((max_len,), -1, dtype=torch.int64, device=dev)
    forced[3] = 1234
    pos = torch.tensor([1], dtype=torch.int32, device=dev)
    token = torch.zeros(1, dtype=torch.int64, device=dev)
    log = torch.full((max_len,), -7, dtype=torch.int64, device=dev)
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    fn = lib.tq4_argmax_advance
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(fn(vp(logits), n, vp(forced), max_len, vp(pos), vp(token), vp(log), max_len, st))
    torch.cuda.synchronize()
    assert int(pos.item()) == 2 and int(token.item()) == want and int(log[2].item()) == want
    _lib.check(fn(vp(logits), n, vp(forced), max_len, vp(pos), vp(token), vp(log), max_len, st))  # forced step
    torch.cuda.synchronize()
    assert int(pos.item()) == 3 and int(token.item()) == 1234 and int(log[3].item()) == 1234
