// Decoder kernels around MatMulNBits (include/tq4_decoder.h): residual RMSNorm, QK-norm + RoPE,
// one-token GQA attention over an f32 KV cache, SwiGLU, and the greedy argmax step. All f32; the
// position and the tokens live in device memory so a decode step replays as one CUDA graph.
#include "../../include/tq4_decoder.h"
#include "internal.cuh"

#include <map>
#include <memory>
#include <mutex>

namespace tq4 {

tq4_status run_gemv_fused(const Weight& w, const float* x, const float* x2, const float* norm_w, float eps,
                          int mode, const float* residual, float* y, cudaStream_t st);

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
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  float* xr = x + blockIdx.x * n;
  float* yr = y + blockIdx.x * n;
  const float* dr = delta ? delta + blockIdx.x * n : nullptr;
  float ss = 0.f;
  if (n <= 8 * 256) {  // the row stays in registers: one memory round trip
    float v[8], wv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = threadIdx.x + 256 * j;
      v[j] = i < n ? xr[i] : 0.f;
      wv[j] = i < n ? w[i] : 0.f;
      if (dr && i < n) v[j] += dr[i];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = threadIdx.x + 256 * j;
      if (dr && i < n) xr[i] = v[j];
      ss = fmaf(v[j], v[j], ss);
    }
    const float inv = 1.f / sqrtf(block_sum<256>(ss, red) / (float)n + eps);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = threadIdx.x + 256 * j;
      if (i < n) yr[i] = v[j] * inv * wv[j];
    }
    return;
  }
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
  pdl_wait();
  pdl_trigger();
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

// One-token GroupQueryAttention, split over positions (flash-decoding). CTA (chunk c, KV head kvh)
// takes positions [32c, 32c + 32) for all G = heads / kv_heads query heads of that KV head, so each
// K/V row is read once per token. A chunk keeps its max m, sum l and unnormalised output
// o = sum_p exp(s_p - m) v_p; the last chunk CTA of a KV head (atomic arrival count) combines them
// in chunk order, so the result does not depend on scheduling. The CTA whose chunk holds the new
// position writes k_new / v_new into the cache; the other chunks never read that row. A CTA first
// copies its chunk of K and V into shared memory with 16-byte loads all in flight together (one
// memory round trip), then works from there.
constexpr int kAttnChunk = 32;
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxGroup = 8;
constexpr int kAttnMaxDim = 256;

__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(
    const float* __restrict__ q, const float* __restrict__ k_new, const float* __restrict__ v_new,
    float* __restrict__ k_cache, float* __restrict__ v_cache, const int32_t* __restrict__ pos,
    float* __restrict__ out, int heads, int kv_heads, int head_dim, int max_len, float scale,
    float* __restrict__ part, int* __restrict__ counters, int chunks_max, const float* __restrict__ q_w,
    const float* __restrict__ k_w, const float* __restrict__ cos_t, const float* __restrict__ sin_t, float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float qs[kAttnMaxGroup * kAttnMaxDim];
  __shared__ float sc[kAttnMaxGroup][kAttnChunk];
  __shared__ float ml[kAttnMaxGroup][2];
  __shared__ int s_last;
  const int G = heads / kv_heads;
  const int c = blockIdx.x, kvh = blockIdx.y;
  const int L = *pos + 1;
  if (L < 1 || L > max_len) {  // position past the cache
    if (threadIdx.x == 0 && c == 0) report(kDevBadArgument);
    return;
  }
  const int nch = (L + kAttnChunk - 1) / kAttnChunk;
  const int p0 = c * kAttnChunk;
  if (p0 >= L) return;
  const int np = min(kAttnChunk, L - p0);
  const int64_t D = head_dim;
  const float* kn = k_new + kvh * D;
  const float* vn = v_new + kvh * D;
  float* kc = k_cache + (int64_t)kvh * max_len * D;
  float* vc = v_cache + (int64_t)kvh * max_len * D;
  const bool has_new = (p0 + np == L);  // this chunk holds position L - 1
  extern __shared__ float4 kv_chunk[];  // K rows [kAttnChunk][D], then V rows
  float* ks = reinterpret_cast<float*>(kv_chunk);
  float* vs = ks + kAttnChunk * D;
  const int D4 = head_dim / 4;
#pragma unroll 8
  for (int i = threadIdx.x; i < np * D4; i += kAttnThreads) {
    const int pi = i / D4, d4 = i - pi * D4;
    const bool nw = (p0 + pi == L - 1);
    const float4* kr = reinterpret_cast<const float4*>(nw ? kn : kc + (int64_t)(p0 + pi) * D);
    const float4* vr = reinterpret_cast<const float4*>(nw ? vn : vc + (int64_t)(p0 + pi) * D);
    reinterpret_cast<float4*>(ks)[i] = kr[d4];
    reinterpret_cast<float4*>(vs)[i] = vr[d4];
  }
  for (int i = threadIdx.x; i < G * head_dim; i += kAttnThreads) qs[i] = q[(int64_t)kvh * G * D + i];
  __syncthreads();
  float* knew_s = has_new ? ks + (L - 1 - p0) * D : nullptr;  // the new key's staged row
  if (q_w) {
    // Qwen3's per-head RMSNorm then rotate-half RoPE at position L - 1 (rms_norm/4,
    // transformer.ex:1056-1069; rotate/4, :558-590), on the query heads and the new key.
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows = G + (has_new ? 1 : 0);
    for (int r = warp; r < rows; r += kAttnThreads / 32) {
      float* v = r < G ? qs + r * D : knew_s;
      const float* w = r < G ? q_w : k_w;
      float ss = 0.f;
      for (int d = lane; d < head_dim; d += 32) ss = fmaf(v[d], v[d], ss);
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float inv = 1.f / sqrtf(ss / (float)head_dim + eps);
      __syncwarp();
      for (int d = lane; d < head_dim; d += 32) v[d] = v[d] * inv * w[d];
    }
    __syncthreads();
    const int half = head_dim / 2;
    const float* cr = cos_t + (int64_t)(L - 1) * half;
    const float* sr = sin_t + (int64_t)(L - 1) * half;
    for (int i = threadIdx.x; i < rows * half; i += kAttnThreads) {
      const int r = i / half, j = i % half;
      float* v = r < G ? qs + r * D : knew_s;
      const float c = cr[j], sn = sr[j];
      const float x1 = v[j], x2 = v[j + half];
      v[j] = x1 * c - x2 * sn;
      v[j + half] = x2 * c + x1 * sn;
    }
    __syncthreads();
  }
  if (has_new)
    for (int d = threadIdx.x; d < head_dim; d += kAttnThreads) {
      kc[(int64_t)(L - 1) * D + d] = knew_s[d];
      vc[(int64_t)(L - 1) * D + d] = vn[d];
    }
  __syncthreads();

  // scores: warp w takes positions w, w + 4, ...; lanes split head_dim
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < np; i += kAttnThreads / 32) {
    const float* kp = ks + i * D;
    float dot[kAttnMaxGroup];
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) dot[g] = 0.f;
    for (int d = lane; d < head_dim; d += 32) {
      const float kv = kp[d];
#pragma unroll
      for (int g = 0; g < kAttnMaxGroup; ++g)
        if (g < G) dot[g] = fmaf(qs[g * head_dim + d], kv, dot[g]);
    }
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) {
      if (g >= G) break;
      float v = dot[g];
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) sc[g][i] = v * scale;
    }
  }
  __syncthreads();
  // chunk softmax statistics: warp w takes heads w, w + 4, ...
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    const float v = lane < np ? sc[g][lane] : -INFINITY;
    float m = v;
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float e = lane < np ? expf(v - m) : 0.f;
    float l = e;
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane < np) sc[g][lane] = e;
    if (lane == 0) {
      ml[g][0] = m;
      ml[g][1] = l;
    }
  }
  __syncthreads();
  // o[g][d] = sum_p e[g][p] v[p][d]
  const int64_t stride_c = (int64_t)G * (D + 2);
  float* my = part + ((int64_t)kvh * chunks_max + c) * stride_c;
  for (int d = threadIdx.x; d < head_dim; d += kAttnThreads) {
    float o[kAttnMaxGroup];
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) o[g] = 0.f;
    for (int i = 0; i < np; ++i) {
      const float vv = vs[i * D + d];
#pragma unroll
      for (int g = 0; g < kAttnMaxGroup; ++g)
        if (g < G) o[g] = fmaf(sc[g][i], vv, o[g]);
    }
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) {
      if (g >= G) break;
      if (nch == 1)
        out[((int64_t)kvh * G + g) * D + d] = o[g] / ml[g][1];
      else
        my[g * (D + 2) + d] = o[g];
    }
  }
  if (nch == 1) return;
  if (threadIdx.x < G) {
    my[threadIdx.x * (D + 2) + D] = ml[threadIdx.x][0];
    my[threadIdx.x * (D + 2) + D + 1] = ml[threadIdx.x][1];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&counters[kvh], 1);
    s_last = (prev == nch - 1);
    if (prev >= nch) report(kDevTimeoutSplitK);  // a counter left non-zero earlier
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* base = part + (int64_t)kvh * chunks_max * stride_c;
  for (int i = threadIdx.x; i < G * head_dim; i += kAttnThreads) {
    const int g = i / head_dim, d = i % head_dim;
    float M = -INFINITY;
    for (int cc = 0; cc < nch; ++cc) M = fmaxf(M, base[cc * stride_c + g * (D + 2) + D]);
    float num = 0.f, den = 0.f;
    for (int cc = 0; cc < nch; ++cc) {
      const float* pc = base + cc * stride_c + g * (D + 2);
      const float w = expf(pc[D] - M);
      num = fmaf(w, pc[d], num);
      den = fmaf(w, pc[D + 1], den);
    }
    out[((int64_t)kvh * G + g) * D + d] = num / den;
  }
  if (threadIdx.x == 0) counters[kvh] = 0;
}

// Per-(device, stream) scratch of the attention partials and arrival counters.
struct AttnScratch {
  DeviceBuffer part, counters;
};
static std::mutex g_attn_mu;
static std::map<std::pair<int, cudaStream_t>, std::unique_ptr<AttnScratch>> g_attn_scratch;

static tq4_status attn_scratch(cudaStream_t st, int64_t part_bytes, int64_t counters, float** part, int** ctr) {
  int dev = 0;
  TQ4_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_attn_mu);
  auto& slot = g_attn_scratch[{dev, st}];
  if (!slot) slot.reset(new AttnScratch());
  if (slot->part.bytes < part_bytes || slot->counters.bytes < counters * 4) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    TQ4_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone) {
      set_error("tq4_attention_decode: first call on a stream (or a larger cache) during stream capture; "
                "call it once before capturing");
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    TQ4_CUDA(cudaStreamSynchronize(st));
    if (slot->part.bytes < part_bytes) TQ4_TRY(slot->part.alloc(part_bytes));
    if (slot->counters.bytes < counters * 4) {
      TQ4_TRY(slot->counters.alloc(counters * 4));
      TQ4_CUDA(cudaMemsetAsync(slot->counters.ptr, 0, counters * 4, st));
    }
  }
  *part = static_cast<float*>(slot->part.ptr);
  *ctr = static_cast<int*>(slot->counters.ptr);
  return TQ4_OK;
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out,
                                int64_t n) {
  pdl_wait();
  pdl_trigger();
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
  pdl_wait();
  pdl_trigger();
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
  TQ4_CUDA(launch_pdl(add_rmsnorm_kernel, dim3((unsigned)rows), dim3(256), 0, static_cast<cudaStream_t>(stream), x,
                      delta, w, y, n, eps));
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
  TQ4_CUDA(launch_pdl(qk_norm_rope_kernel, dim3(heads + kv_heads), dim3(128), 0, static_cast<cudaStream_t>(stream),
                      q, k, q_w, k_w, cos_table, sin_table, pos, heads, head_dim, max_pos, eps));
  return TQ4_OK;
}

namespace {
struct RopeArgs {
  const float* q_w = nullptr;
  const float* k_w = nullptr;
  const float* cos_t = nullptr;
  const float* sin_t = nullptr;
  float eps = 0.f;
};
tq4_status attention_impl(const float* q, const float* k_new, const float* v_new, float* k_cache, float* v_cache,
                          const int32_t* pos, float* out, int heads, int kv_heads, int head_dim, int max_len,
                          void* stream, const RopeArgs& rope);
}  // namespace

tq4_status tq4_attention_decode(const float* q, const float* k_new, const float* v_new,
                                float* k_cache, float* v_cache, const int32_t* pos, float* out,
                                int heads, int kv_heads, int head_dim, int max_len, void* stream) {
  clear_error();
  return attention_impl(q, k_new, v_new, k_cache, v_cache, pos, out, heads, kv_heads, head_dim, max_len, stream,
                        RopeArgs{});
}

tq4_status tq4_attention_decode_rope(const float* q, const float* k_new, const float* v_new, const float* q_w,
                                     const float* k_w, const float* cos_table, const float* sin_table, float eps,
                                     float* k_cache, float* v_cache, const int32_t* pos, float* out, int heads,
                                     int kv_heads, int head_dim, int max_len, void* stream) {
  clear_error();
  if (!q_w || !k_w || !cos_table || !sin_table || (head_dim & 1)) {
    set_error("tq4_attention_decode_rope: null norm weight / table, or odd head_dim");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  RopeArgs r;
  r.q_w = q_w;
  r.k_w = k_w;
  r.cos_t = cos_table;
  r.sin_t = sin_table;
  r.eps = eps;
  return attention_impl(q, k_new, v_new, k_cache, v_cache, pos, out, heads, kv_heads, head_dim, max_len, stream, r);
}

tq4_status tq4_matmul_fused(const tq4_weight* w, const float* x, const float* x2, const float* norm_w, float eps,
                            int prologue, const float* residual, float* y, void* stream) {
  clear_error();
  if (!w || !x || !y || prologue < 0 || prologue > 2 || (prologue == 1 && !norm_w) || (prologue == 2 && !x2)) {
    set_error("tq4_matmul_fused: bad arguments (RMSNorm needs norm_w, SwiGLU needs x2)");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceGuard guard(w->device);
  return run_gemv_fused(*w, x, x2, norm_w, eps, prologue, residual, y, static_cast<cudaStream_t>(stream));
}

namespace {
tq4_status attention_impl(const float* q, const float* k_new, const float* v_new, float* k_cache, float* v_cache,
                          const int32_t* pos, float* out, int heads, int kv_heads, int head_dim, int max_len,
                          void* stream, const RopeArgs& rope) {
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !pos || !out || heads <= 0 || kv_heads <= 0 ||
      heads % kv_heads || heads / kv_heads > kAttnMaxGroup || head_dim <= 0 || head_dim > kAttnMaxDim ||
      (head_dim & 3) || max_len <= 0 || kv_heads > 65535 ||
      ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
        reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)) {
    set_error("tq4_attention_decode: bad arguments (heads a multiple of kv_heads, at most %d query heads per "
              "KV head, head_dim a multiple of 4 and <= %d, K/V pointers 16-byte aligned)",
              kAttnMaxGroup, kAttnMaxDim);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = heads / kv_heads;
  const int chunks = (max_len + kAttnChunk - 1) / kAttnChunk;
  float* part = nullptr;
  int* ctr = nullptr;
  TQ4_TRY(attn_scratch(st, (int64_t)kv_heads * chunks * G * (head_dim + 2) * 4, kv_heads, &part, &ctr));
  const size_t dyn = (size_t)2 * kAttnChunk * head_dim * sizeof(float);
  static bool attr_set = false;
  if (!attr_set) {
    TQ4_CUDA(cudaFuncSetAttribute(attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  2 * kAttnChunk * kAttnMaxDim * (int)sizeof(float)));
    attr_set = true;
  }
  TQ4_CUDA(launch_pdl(attention_decode_kernel, dim3(chunks, kv_heads), dim3(kAttnThreads), dyn, st, q, k_new, v_new,
                      k_cache, v_cache, pos, out, heads, kv_heads, head_dim, max_len, 1.f / sqrtf((float)head_dim),
                      part, ctr, chunks, rope.q_w, rope.k_w, rope.cos_t, rope.sin_t, rope.eps));
  return TQ4_OK;
}
}  // namespace

tq4_status tq4_silu_mul(const float* gate, const float* up, float* out, int64_t n, void* stream) {
  clear_error();
  if (!gate || !up || !out || n < 0) {
    set_error("tq4_silu_mul: bad arguments");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (n == 0) return TQ4_OK;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 1024);
  TQ4_CUDA(launch_pdl(silu_mul_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), gate, up, out, n));
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
  TQ4_CUDA(launch_pdl(argmax_advance_kernel, dim3(1), dim3(1024), 0, static_cast<cudaStream_t>(stream), logits, n,
                      forced, forced_len, pos, token, log, log_len));
  return TQ4_OK;
}

}  // extern "C"
