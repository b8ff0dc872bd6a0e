/*
 * tq4 decoder kernels: the operators around MatMulNBits in a q4 decoder (Qwen3-style), in f32.
 * They serve the decode-throughput configuration of this build; each cites the reference operator
 * whose arithmetic it follows (georgeguimaraes/transmuter 2.0.0, lib/transmuter/ops/transformer.ex).
 * All pointers are device pointers; positions and tokens live in device memory so that a decode
 * step can be captured once in a CUDA graph and replayed.
 */
#ifndef TQ4_DECODER_H
#define TQ4_DECODER_H

#include "tq4.h"

#ifdef __cplusplus
extern "C" {
#endif

/* SkipSimplifiedLayerNormalization (transformer.ex:297-300) and rms_norm/4 (:1056-1069):
 * if delta != NULL, x += delta (the residual stream, in place); then
 * y = x * rsqrt(mean(x^2) + eps) * w for each of `rows` rows of n values. */
tq4_status tq4_add_rmsnorm(float* x, const float* delta, const float* w, float* y, int64_t rows,
                           int64_t n, float eps, void* stream);

/* The per-head RMSNorm of Qwen3's query/key (rms_norm/4 over head_dim) followed by
 * RotaryEmbedding, rotate-half layout (rotate/4, transformer.ex:558-590, interleaved = 0), at the
 * position *pos: q [heads][head_dim] and k [kv_heads][head_dim] in place. cos/sin are
 * [max_pos][head_dim/2] tables. A *pos outside [0, max_pos) leaves q/k untouched and sets the
 * device status (tq4_device_status). */
tq4_status tq4_qk_norm_rope(float* q, float* k, const float* q_w, const float* k_w,
                            const float* cos_table, const float* sin_table, const int32_t* pos,
                            int max_pos, int heads, int kv_heads, int head_dim, float eps,
                            void* stream);

/* GroupQueryAttention for one new token (transformer.ex:106-175, one query row, causal, no
 * window): writes k_new/v_new at *pos of the f32 caches [kv_heads][max_len][head_dim], then
 * out[h] = softmax(q[h] . K[h/g][0..pos] * scale) . V[h/g][0..pos], g = heads / kv_heads,
 * scale = 1/sqrt(head_dim) (:1089-1094). A *pos outside [0, max_len) writes nothing and sets the
 * device status. */
tq4_status tq4_attention_decode(const float* q, const float* k_new, const float* v_new,
                                float* k_cache, float* v_cache, const int32_t* pos, float* out,
                                int heads, int kv_heads, int head_dim, int max_len, void* stream);

/* tq4_attention_decode with Qwen3's per-head RMSNorm (weights q_w / k_w over head_dim, eps) and
 * rotate-half RoPE at *pos (cos/sin tables [max_len][head_dim/2]) applied to q and k_new first,
 * as tq4_qk_norm_rope would: the normalised, rotated key is the one written into the cache.
 * q and k_new are read, not modified. This is the decode step's form: the cache rows before *pos
 * are read while the previous kernel on the stream may still run (programmatic dependent
 * launch), so they must be complete before that kernel started, as in a decode loop where
 * earlier steps wrote them (the row at *pos comes from k_new / v_new). */
tq4_status tq4_attention_decode_rope(const float* q, const float* k_new, const float* v_new,
                                     const float* q_w, const float* k_w, const float* cos_table,
                                     const float* sin_table, float eps, float* k_cache,
                                     float* v_cache, const int32_t* pos, float* out, int heads,
                                     int kv_heads, int head_dim, int max_len, void* stream);

/* A decode-step projection through a MatMulNBits handle (M = 1, f32 in and out; the handle's
 * weight 4-bit with block_size <= 128):
 *   y[n] = residual[n] + (W . a)[n],  a = prologue(x)
 * prologue 0: a = x; 1: a = RMSNorm(x) = x * rsqrt(mean(x^2) + eps) * norm_w
 * (SkipSimplifiedLayerNormalization / rms_norm/4, transformer.ex:290-300,1056-1069); 2: SwiGLU,
 * a = silu(x) * x2 (x and x2 of K values each). residual may be NULL, or equal to y (the
 * decoder's residual stream updated in place). The prologue runs while the GEMV stages its
 * activations, so the normalised row is never written to memory. */
tq4_status tq4_matmul_fused(const tq4_weight* w, const float* x, const float* x2,
                            const float* norm_w, float eps, int prologue, const float* residual,
                            float* y, void* stream);

/* SwiGLU: out[i] = silu(gate[i]) * up[i], silu(x) = x / (1 + exp(-x)). */
tq4_status tq4_silu_mul(const float* gate, const float* up, float* out, int64_t n, void* stream);

/* Greedy step bookkeeping: next = argmax(logits[0..n)) (lowest index on ties), unless
 * *pos + 1 < forced_len and forced[*pos + 1] >= 0, in which case next = forced[*pos + 1] (a
 * prompt token; -1 marks a free position, so one captured graph serves prompts of any length).
 * Then log[*pos + 1] = next (when *pos + 1 < log_len), *token = next and *pos += 1. */
tq4_status tq4_argmax_advance(const float* logits, int64_t n, const int64_t* forced,
                              int forced_len, int32_t* pos, int64_t* token, int64_t* log,
                              int log_len, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TQ4_DECODER_H */
