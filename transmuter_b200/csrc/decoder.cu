// Decoder kernels around MatMulNBits (include/tq4_decoder.h): residual RMSNorm, QK-norm + RoPE,
// one-token GQA attention over an f32 KV cache, SwiGLU, and the greedy argmax step. All f32; the
// position and the tokens live in device memory so a decode step replays as one CUDA graph.
#include "../../include/tq4_decoder.h"
#include "internal.cuh"

namespace tq4 {

// Deterministic block sum (fixed shuffle tree, then warp order).
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float total = 0.f;
  for (int w = 0; w < THREADS / 32; ++w) total += red[w];
  __syncthreads();
  return total;
}

template <int THREADS>
__device__ __forceinline__ float block_max(float v, float* red) {
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
  for (int w = 1; w < THREADS / 32; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

// rms_norm/4 (transformer.ex:1056-1069) with the residual add of SkipSimplifiedLayerNormalization.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                                          const float* __restrict__ w, float* __restrict__ y,
                                                          int64_t n, float eps) {
  __shared__ float red[8];
  float* xr = x + blockIdx.x * n;
  float* yr = y + blockIdx.x * n;
  const float* dr = delta ? delta + blockIdx.x * n : nullptr;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += 256) {
    float v = xr[i];
    if (dr) {
      v += dr[i];
      xr[i] = v;
    }
    ss = fmaf(v, v, ss);
  }
  const float mean = block_sum<256>(ss, red) / (float)n;
  const float inv = 1.f / sqrtf(mean + eps);
  for (int64_t i = threadIdx.x; i < n; i += 256) yr[i] = xr[i] * inv * w[i];
}

// Per-head RMSNorm, then rotate-half RoPE at *pos (rotate/4, transformer.ex:558-590).
__global__ void __launch_bounds__(128) qk_norm_rope_kernel(float* __restrict__ q, float* __restrict__ k,
                                                           const float* __restrict__ q_w, const float* __restrict__ k_w,
                                                           const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                                           const int32_t* __restrict__ pos, int heads, int head_dim,
                                                           int max_pos, float eps) {
  __shared__ float red[4];
  __shared__ float buf[512];
  const int h = blockIdx.x;
  const int64_t p = *pos;
  if (p < 0 || p >= max_pos) {  // position past the tables: leave q/k as they are, flag it
    if (threadIdx.x == 0) report(kDevBadArgument);
    return;
  }
  float* v = h < heads ? q + (int64_t)h * head_dim : k + (int64_t)(h - heads) * head_dim;
  const float* w = h < heads ? q_w : k_w;
  float ss = 0.f;
  for (int i = threadIdx.x; i < head_dim; i += 128) {
    const float x = v[i];
    buf[i] = x;
    ss = fmaf(x, x, ss);
  }
  const float inv = 1.f / sqrtf(block_sum<128>(ss, red) / (float)head_dim + eps);
  for (int i = threadIdx.x; i < head_dim; i += 128) buf[i] = buf[i] * inv * w[i];
  __syncthreads();
  const int half = head_dim / 2;
  for (int i = threadIdx.x; i < half; i += 128) {
    const float c = cos_t[p * half + i], s = sin_t[p * half + i];
    const float x1 = buf[i], x2 = buf[i + half];
    v[i] = x1 * c - x2 * s;
    v[i + half] = x2 * c + x1 * s;
  }
}

// One query row per head; the CTA of the first query head of each KV group also writes the new
// key / value into the cache (the other heads read the new ones from k_new / v_new).
__global__ void __launch_bounds__(128) attention_decode_kernel(const float* __restrict__ q, const float* __restrict__ k_new,
                                                               const float* __restrict__ v_new, float* __restrict__ k_cache,
                                                               float* __restrict__ v_cache, const int32_t* __restrict__ pos,
                                                               float* __restrict__ out, int heads, int kv_heads,
                                                               int head_dim, int max_len, float scale) {
  extern __shared__ float sm[];  // q [head_dim], scores [max_len]
  __shared__ float red[4];
  float* qs = sm;
  float* sc = sm + head_dim;
  const int h = blockIdx.x;
  const int group = heads / kv_heads;
  const int kvh = h / group;
  const int L = *pos + 1;
  if (L < 1 || L > max_len) {  // position past the cache
    if (threadIdx.x == 0) report(kDevBadArgument);
    return;
  }
  const float* kn = k_new + (int64_t)kvh * head_dim;
  const float* vn = v_new + (int64_t)kvh * head_dim;
  float* kc = k_cache + (int64_t)kvh * max_len * head_dim;
  float* vc = v_cache + (int64_t)kvh * max_len * head_dim;
  for (int d = threadIdx.x; d < head_dim; d += 128) {
    qs[d] = q[(int64_t)h * head_dim + d];
    if (h % group == 0) {
      kc[(int64_t)(L - 1) * head_dim + d] = kn[d];
      vc[(int64_t)(L - 1) * head_dim + d] = vn[d];
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int p = warp; p < L; p += 4) {
    const float* kp = (p == L - 1) ? kn : kc + (int64_t)p * head_dim;
    float dot = 0.f;
    for (int d = lane; d < head_dim; d += 32) dot = fmaf(qs[d], kp[d], dot);
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    if (lane == 0) sc[p] = dot * scale;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int p = threadIdx.x; p < L; p += 128) mx = fmaxf(mx, sc[p]);
  mx = block_max<128>(mx, red);
  float sum = 0.f;
  for (int p = threadIdx.x; p < L; p += 128) {
    const float e = expf(sc[p] - mx);
    sc[p] = e;
    sum += e;
  }
  sum = block_sum<128>(sum, red);
  const float inv = 1.f / sum;
  for (int d = threadIdx.x; d < head_dim; d += 128) {
    float o = 0.f;
    for (int p = 0; p < L; ++p) {
      const float vv = (p == L - 1) ? vn[d] : vc[(int64_t)p * head_dim + d];
      o = fmaf(sc[p], vv, o);
    }
    out[(int64_t)h * head_dim + d] = o * inv;
  }
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out,
                                int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = g[i];
    out[i] = x / (1.f + expf(-x)) * u[i];
  }
}

// Greedy argmax (lowest index among equal maxima; NaN never wins) and the step bookkeeping.
__global__ void __launch_bounds__(1024) argmax_advance_kernel(const float* __restrict__ logits, int64_t n,
                                                              const int64_t* __restrict__ forced, int forced_len,
                                                              int32_t* __restrict__ pos, int64_t* __restrict__ token,
                                                              int64_t* __restrict__ log, int log_len) {
  __shared__ float bv[32];
  __shared__ int64_t bi[32];
  float best = -INFINITY;
  int64_t idx = n;
  for (int64_t i = threadIdx.x; i < n; i += 1024) {
    const float v = logits[i];
    if (v > best || (v == best && i < idx)) {
      best = v;
      idx = i;
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, off);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 32; ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
        best = bv[w];
        idx = bi[w];
      }
    const int next_pos = *pos + 1;
    const int64_t f = next_pos < forced_len ? forced[next_pos] : -1;
    const int64_t next = f >= 0 ? f : (idx < n ? idx : 0);
    if (next_pos < log_len) log[next_pos] = next;
    *token = next;
    *pos = next_pos;
  }
}

}  // namespace tq4

using namespace tq4;

extern "C" {

tq4_status tq4_add_rmsnorm(float* x, const float* delta, const float* w, float* y, int64_t rows,
                           int64_t n, float eps, void* stream) {
  clear_error();
  if (!x || !w || !y || rows < 0 || n <= 0) {
    set_error("tq4_add_rmsnorm: bad arguments");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (rows == 0) return TQ4_OK;
  add_rmsnorm_kernel<<<(unsigned)rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, delta, w, y, n, eps);
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

tq4_status tq4_qk_norm_rope(float* q, float* k, const float* q_w, const float* k_w,
                            const float* cos_table, const float* sin_table, const int32_t* pos,
                            int max_pos, int heads, int kv_heads, int head_dim, float eps, void* stream) {
  clear_error();
  if (!q || !k || !q_w || !k_w || !cos_table || !sin_table || !pos || max_pos <= 0 || heads <= 0 ||
      kv_heads <= 0 || head_dim <= 0 || head_dim > 512 || (head_dim & 1)) {
    set_error("tq4_qk_norm_rope: bad arguments (head_dim must be even and <= 512)");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  qk_norm_rope_kernel<<<heads + kv_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, q_w, k_w, cos_table, sin_table, pos, heads, head_dim, max_pos, eps);
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

tq4_status tq4_attention_decode(const float* q, const float* k_new, const float* v_new,
                                float* k_cache, float* v_cache, const int32_t* pos, float* out,
                                int heads, int kv_heads, int head_dim, int max_len, void* stream) {
  clear_error();
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !pos || !out || heads <= 0 || kv_heads <= 0 ||
      heads % kv_heads || head_dim <= 0 || max_len <= 0 || (size_t)(head_dim + max_len) * 4 > 200 * 1024) {
    set_error("tq4_attention_decode: bad arguments");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  const size_t smem = (size_t)(head_dim + max_len) * sizeof(float);
  if (smem > 48 * 1024) TQ4_CUDA(cudaFuncSetAttribute(attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  attention_decode_kernel<<<heads, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      q, k_new, v_new, k_cache, v_cache, pos, out, heads, kv_heads, head_dim, max_len,
      1.f / sqrtf((float)head_dim));
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

tq4_status tq4_silu_mul(const float* gate, const float* up, float* out, int64_t n, void* stream) {
  clear_error();
  if (!gate || !up || !out || n < 0) {
    set_error("tq4_silu_mul: bad arguments");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (n == 0) return TQ4_OK;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 1024);
  silu_mul_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(gate, up, out, n);
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

tq4_status tq4_argmax_advance(const float* logits, int64_t n, const int64_t* forced,
                              int forced_len, int32_t* pos, int64_t* token, int64_t* log,
                              int log_len, void* stream) {
  clear_error();
  if (!logits || n <= 0 || !pos || !token || (forced_len > 0 && !forced) || (log_len > 0 && !log)) {
    set_error("tq4_argmax_advance: bad arguments");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  argmax_advance_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(logits, n, forced, forced_len,
                                                                          pos, token, log, log_len);
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

}  // extern "C"
