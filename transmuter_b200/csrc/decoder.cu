// Decoder kernels around MatMulNBits (include/tq4_decoder.h): residual RMSNorm, QK-norm + RoPE,
// one-token GQA attention over an f32 KV cache, SwiGLU, and the greedy argmax step. All f32; the
// position and the tokens live in device memory so a decode step replays as one CUDA graph.
#include "../../include/tq4_decoder.h"
#include "internal.cuh"
#include "sm100.cuh"

#include <algorithm>

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

// One-token GroupQueryAttention, split over positions (flash-decoding) within a thread-block
// cluster. The C CTAs of KV head kvh (grid (C, kv_heads), cluster (C, 1, 1)) take 32-position
// chunks in turn: rank r owns chunks r, r + C, ... and keeps, for each of the G = heads / kv_heads
// query heads, a running max m, sum l and unnormalised output o = sum_p exp(s_p - m) v_p (online
// softmax over its chunks). The ranks then combine (m, l, o) through distributed shared memory in
// rank order, so the result does not depend on scheduling, and each rank writes a slice of the
// output. The rank whose chunk holds position L - 1 writes k_new / v_new into the cache; every
// chunk sees the new row from shared memory.
//
// Latency is the whole cost at decode sizes, so the memory round trips are few: the first chunk's
// K and V rows travel as two bulk copies issued before the position is known (the rows of chunk r
// lie inside the cache whatever the position; rows at or past L are never used), together with q,
// k_new, v_new and the norm weights; only the RoPE table row waits for the position.
constexpr int kAttnChunk = 32;
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxGroup = 8;
constexpr int kAttnMaxDim = 256;
constexpr int kAttnMaxCluster = 8;

template <int G>  // query heads per KV head
__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(
    const float* __restrict__ q, const float* __restrict__ k_new, const float* __restrict__ v_new,
    float* __restrict__ k_cache, float* __restrict__ v_cache, const int32_t* __restrict__ pos,
    float* __restrict__ out, int heads, int kv_heads, int head_dim, int max_len, float scale,
    const float* __restrict__ q_w, const float* __restrict__ k_w, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, float eps, int early) {
  __shared__ __align__(16) float qs[kAttnMaxGroup * kAttnMaxDim];
  __shared__ __align__(16) float kn_s[kAttnMaxDim];
  __shared__ __align__(16) float vn_s[kAttnMaxDim];
  __shared__ __align__(16) float qw_s[kAttnMaxDim];
  __shared__ __align__(16) float kw_s[kAttnMaxDim];
  __shared__ __align__(16) float cs_s[kAttnMaxDim / 2];
  __shared__ __align__(16) float sn_s[kAttnMaxDim / 2];
  __shared__ float sc[kAttnMaxGroup][kAttnChunk];
  __shared__ float spart[kAttnMaxGroup][kAttnChunk];  // partial scores of the D slices
  __shared__ float ml[kAttnMaxGroup][2];  // running max, running sum
  __shared__ float alpha_s[kAttnMaxGroup];
  __shared__ float part[kAttnMaxGroup * (kAttnMaxDim + 2)];  // o[g][0..D), m, l: read by the cluster
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_abort;
  extern __shared__ float4 kv_chunk[];  // K rows [kAttnChunk][D], then V rows

  const int D = head_dim, D4 = head_dim / 4;
  const int C = (int)gridDim.x;  // the cluster spans x
  const int r = (int)cluster_ctarank(), kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* ks = reinterpret_cast<float*>(kv_chunk);
  float* vs = ks + kAttnChunk * D;
  const uint32_t bar_a = smem_u32(&bar);
  float* kc = k_cache + (int64_t)kvh * max_len * D;
  float* vc = v_cache + (int64_t)kvh * max_len * D;

  // Trip 1: the first chunk's cache rows (bulk copies). With `early` they are issued before the
  // wait for the previous kernel: the caller guarantees that the rows before this step's position
  // were complete before that kernel started (in a decode step, earlier steps wrote them and every
  // kernel waits for the one before it), and the row of this step's position is taken from
  // k_new / v_new below.
  const int rows0 = min(kAttnChunk, max_len - r * kAttnChunk);  // >= 1: C <= ceil(max_len / 32)
  if (!early) pdl_wait();
  if (tid == 0) {
    s_abort = 0;
    mbar_init(bar_a, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async_smem();
    const uint32_t bytes = (uint32_t)(rows0 * D * 4);
    mbar_expect_tx(bar_a, 2 * bytes);
    bulk_load(smem_u32(ks), kc + (int64_t)r * kAttnChunk * D, bytes, bar_a);
    bulk_load(smem_u32(vs), vc + (int64_t)r * kAttnChunk * D, bytes, bar_a);
  }
  if (early) pdl_wait();
  pdl_trigger();
  // Then the position, q, the new row and the norm weights.
  const int L = *pos + 1;
  const float4* q4 = reinterpret_cast<const float4*>(q + (int64_t)kvh * G * D);
  float4 qr[kAttnMaxGroup * kAttnMaxDim / 4 / kAttnThreads];
#pragma unroll
  for (int j = 0; j < kAttnMaxGroup * kAttnMaxDim / 4 / kAttnThreads; ++j) {
    const int i = tid + j * kAttnThreads;
    if (i < G * D4) qr[j] = q4[i];
  }
  float4 knr, vnr, qwr, kwr;
  if (tid < D4) {
    knr = reinterpret_cast<const float4*>(k_new + (int64_t)kvh * D)[tid];
    vnr = reinterpret_cast<const float4*>(v_new + (int64_t)kvh * D)[tid];
    if (q_w) {
      qwr = reinterpret_cast<const float4*>(q_w)[tid];
      kwr = reinterpret_cast<const float4*>(k_w)[tid];
    }
  }
  const bool valid = L >= 1 && L <= max_len;  // the same for every CTA
  const int half = D / 2;
  float cv = 0.f, sv = 0.f;
  if (q_w && valid && tid < half) {  // trip 2: the RoPE table row of position L - 1
    cv = cos_t[(int64_t)(L - 1) * half + tid];
    sv = sin_t[(int64_t)(L - 1) * half + tid];
  }
#pragma unroll
  for (int j = 0; j < kAttnMaxGroup * kAttnMaxDim / 4 / kAttnThreads; ++j) {
    const int i = tid + j * kAttnThreads;
    if (i < G * D4) reinterpret_cast<float4*>(qs)[i] = qr[j];
  }
  if (tid < D4) {
    reinterpret_cast<float4*>(kn_s)[tid] = knr;
    reinterpret_cast<float4*>(vn_s)[tid] = vnr;
    if (q_w) {
      reinterpret_cast<float4*>(qw_s)[tid] = qwr;
      reinterpret_cast<float4*>(kw_s)[tid] = kwr;
    }
  }
  if (tid < half) {
    cs_s[tid] = cv;
    sn_s[tid] = sv;
  }
  if (tid < G) {
    ml[tid][0] = -INFINITY;
    ml[tid][1] = 0.f;
  }
  __syncthreads();
  if (!valid) {  // position past the cache: every CTA sees it, none writes anything
    if (tid == 0 && r == 0 && kvh == 0) report(kDevBadArgument);
    mbar_drain(bar_a, 0);
    return;
  }

  if (q_w && D == 128) {
    // Qwen3's per-head RMSNorm then rotate-half RoPE at position L - 1 (rms_norm/4,
    // transformer.ex:1056-1069; rotate/4, :558-590), on the G query heads and the new key; a warp
    // per row, lane l holding d = 4l .. 4l + 3 (its rotation partner d -/+ 64 is lane l ^ 16).
    for (int row = warp; row <= G; row += kAttnThreads / 32) {
      float* v = row < G ? qs + row * D : kn_s;
      const float* w = row < G ? qw_s : kw_s;
      float4 x = reinterpret_cast<const float4*>(v)[lane];
      float ss = fmaf(x.w, x.w, fmaf(x.z, x.z, fmaf(x.y, x.y, x.x * x.x)));
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float inv = 1.f / sqrtf(ss / (float)D + eps);
      const float4 wv = reinterpret_cast<const float4*>(w)[lane];
      x = make_float4(x.x * inv * wv.x, x.y * inv * wv.y, x.z * inv * wv.z, x.w * inv * wv.w);
      float4 pr;
      pr.x = __shfl_xor_sync(0xffffffffu, x.x, 16);
      pr.y = __shfl_xor_sync(0xffffffffu, x.y, 16);
      pr.z = __shfl_xor_sync(0xffffffffu, x.z, 16);
      pr.w = __shfl_xor_sync(0xffffffffu, x.w, 16);
      const float4 c = reinterpret_cast<const float4*>(cs_s)[lane & 15];
      const float4 sn = reinterpret_cast<const float4*>(sn_s)[lane & 15];
      if (lane < 16)  // x = x1 (d < 64), pr = x2: x1 c - x2 s
        x = make_float4(x.x * c.x - pr.x * sn.x, x.y * c.y - pr.y * sn.y, x.z * c.z - pr.z * sn.z,
                        x.w * c.w - pr.w * sn.w);
      else  // x = x2, pr = x1: x2 c + x1 s
        x = make_float4(x.x * c.x + pr.x * sn.x, x.y * c.y + pr.y * sn.y, x.z * c.z + pr.z * sn.z,
                        x.w * c.w + pr.w * sn.w);
      reinterpret_cast<float4*>(v)[lane] = x;
    }
    __syncthreads();
  } else if (q_w) {
    // the same for other head sizes: a warp per row, lanes striding over d
    for (int row = warp; row <= G; row += kAttnThreads / 32) {
      float* v = row < G ? qs + row * D : kn_s;
      const float* w = row < G ? qw_s : kw_s;
      float ss = 0.f;
      for (int d = lane; d < D; d += 32) ss = fmaf(v[d], v[d], ss);
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float inv = 1.f / sqrtf(ss / (float)D + eps);
      __syncwarp();
      for (int d = lane; d < D; d += 32) v[d] = v[d] * inv * w[d];
      __syncwarp();
      for (int j = lane; j < half; j += 32) {
        const float c = cs_s[j], sn = sn_s[j];
        const float x1 = v[j], x2 = v[j + half];
        v[j] = x1 * c - x2 * sn;
        v[j + half] = x2 * c + x1 * sn;
      }
    }
    __syncthreads();
  }

  // This rank's chunks, each folded into the running (m, l, o) of every query head.
  constexpr int kDPer = kAttnMaxDim / kAttnThreads;  // output columns per thread
  float o[kDPer][kAttnMaxGroup];
#pragma unroll
  for (int j = 0; j < kDPer; ++j)
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) o[j][g] = 0.f;
  uint32_t parity = 0;
  mbar_wait(bar_a, 0, &s_abort, kDevTimeoutAttn);  // the first chunk's copies, used or not
  for (int c = r; c * kAttnChunk < L; c += C) {
    const int p0 = c * kAttnChunk, np = min(kAttnChunk, L - p0);
    if (c != r) {  // a later chunk (contexts past 32 * C positions): the buffer is free again
      __syncthreads();
      parity ^= 1u;
      if (tid == 0) {
        fence_proxy_async_smem();
        const uint32_t bytes = (uint32_t)(np * D * 4);
        mbar_expect_tx(bar_a, 2 * bytes);
        bulk_load(smem_u32(ks), kc + (int64_t)p0 * D, bytes, bar_a);
        bulk_load(smem_u32(vs), vc + (int64_t)p0 * D, bytes, bar_a);
      }
      mbar_wait(bar_a, parity, &s_abort, kDevTimeoutAttn);
    }
    if (p0 + np == L)  // this chunk holds the new position: its row comes from k_new / v_new
      for (int d = tid; d < D; d += kAttnThreads) {
        ks[(np - 1) * D + d] = kn_s[d];
        vs[(np - 1) * D + d] = vn_s[d];
      }
    __syncthreads();
    // scores: lane = position (rows past np are computed on whatever the buffer holds and never
    // used); a warp takes one (head, slice of D) pair: G < 4 splits D into 4 / G slices so all
    // four warps work. K rows and q are read as float4 in a lane-rotated chunk order, so the 8
    // lanes of a quarter warp read 8 different 16-byte bank groups; no shuffles.
    {
      constexpr int NS = G >= 4 ? 1 : 4 / G;
      for (int task = warp; task < G * NS; task += kAttnThreads / 32) {
        const int g = task % G, sl = task / G;
        const int c0 = sl * D4 / NS, len = (sl + 1) * D4 / NS - c0;
        if (len == 0) {  // head_dim below 16: fewer chunks than slices
          spart[task][lane] = 0.f;
          continue;
        }
        const float4* kp = reinterpret_cast<const float4*>(ks + lane * D);
        const float4* qp = reinterpret_cast<const float4*>(qs + g * D);
        float a0 = 0.f, a1 = 0.f;
        int c = c0 + lane % len;
        for (int j = 0; j < len; ++j) {
          const float4 kv = kp[c], qv = qp[c];
          a0 = fmaf(qv.x, kv.x, a0);
          a1 = fmaf(qv.y, kv.y, a1);
          a0 = fmaf(qv.z, kv.z, a0);
          a1 = fmaf(qv.w, kv.w, a1);
          if (++c == c0 + len) c = c0;
        }
        spart[task][lane] = a0 + a1;
      }
      __syncthreads();
      for (int i = tid; i < G * kAttnChunk; i += kAttnThreads) {
        const int g = i / kAttnChunk, pp = i % kAttnChunk;
        float v = spart[g][pp];
#pragma unroll
        for (int sl = 1; sl < NS; ++sl) v += spart[sl * G + g][pp];
        sc[g][pp] = v * scale;
      }
    }
    __syncthreads();
    // online softmax statistics: warp w takes heads w, w + 4, ...
    for (int g = warp; g < G; g += kAttnThreads / 32) {
      const float v = lane < np ? sc[g][lane] : -INFINITY;
      float mc = v;
      for (int off = 16; off > 0; off >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
      const float m_old = ml[g][0];
      const float m_new = fmaxf(m_old, mc);
      const float e = lane < np ? expf(v - m_new) : 0.f;
      float l = e;
      for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane < np) sc[g][lane] = e;
      __syncwarp();
      if (lane == 0) {
        const float alpha = expf(m_old - m_new);  // 0 on the first chunk (m_old = -inf)
        alpha_s[g] = alpha;
        ml[g][0] = m_new;
        ml[g][1] = ml[g][1] * alpha + l;
      }
    }
    __syncthreads();
    // o[g][d] = alpha[g] o[g][d] + sum_p e[g][p] v[p][d]
#pragma unroll
    for (int j = 0; j < kDPer; ++j) {
      const int d = tid + j * kAttnThreads;
      if (d < D) {
        float acc[kAttnMaxGroup];
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g) acc[g] = 0.f;
#pragma unroll 4
        for (int i = 0; i < np; ++i) {
          const float vv = vs[i * D + d];
#pragma unroll
          for (int g = 0; g < kAttnMaxGroup; ++g)
            if (g < G) acc[g] = fmaf(sc[g][i], vv, acc[g]);
        }
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g)
          if (g < G) o[j][g] = fmaf(o[j][g], alpha_s[g], acc[g]);
      }
    }
  }
  // The rank that holds position L - 1 stores the new row (its chunk's bulk copies have landed).
  if (((L - 1) / kAttnChunk) % C == r)
    for (int d = tid; d < D; d += kAttnThreads) {
      kc[(int64_t)(L - 1) * D + d] = kn_s[d];
      vc[(int64_t)(L - 1) * D + d] = vn_s[d];
    }
  // Leave this rank's (o, m, l) for the cluster.
#pragma unroll
  for (int j = 0; j < kDPer; ++j) {
    const int d = tid + j * kAttnThreads;
    if (d < D)
#pragma unroll
      for (int g = 0; g < kAttnMaxGroup; ++g)
        if (g < G) part[g * (D + 2) + d] = o[j][g];
  }
  if (tid < G) {
    part[tid * (D + 2) + D] = ml[tid][0];
    part[tid * (D + 2) + D + 1] = ml[tid][1];
  }
  cluster_sync_all();
  // Combine in rank order; rank r writes outputs r * 128 + tid, then every C * 128 further.
  for (int i = r * kAttnThreads + tid; i < G * D; i += C * kAttnThreads) {
    const int g = i / D, d = i - g * D;
    float mr[kAttnMaxCluster], lr[kAttnMaxCluster], orr[kAttnMaxCluster];
#pragma unroll
    for (int cc = 0; cc < kAttnMaxCluster; ++cc)
      if (cc < C) {
        mr[cc] = ld_cluster_f32(part + g * (D + 2) + D, (unsigned)cc);
        lr[cc] = ld_cluster_f32(part + g * (D + 2) + D + 1, (unsigned)cc);
        orr[cc] = ld_cluster_f32(part + g * (D + 2) + d, (unsigned)cc);
      }
    float M = -INFINITY;
#pragma unroll
    for (int cc = 0; cc < kAttnMaxCluster; ++cc)
      if (cc < C) M = fmaxf(M, mr[cc]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int cc = 0; cc < kAttnMaxCluster; ++cc)
      if (cc < C) {
        const float w = expf(mr[cc] - M);  // 0 for a rank without positions (m = -inf)
        num = fmaf(w, orr[cc], num);
        den = fmaf(w, lr[cc], den);
      }
    out[((int64_t)kvh * G + g) * D + d] = num / den;
  }
  if (s_abort) mbar_drain(bar_a, parity);  // a copy that timed out: give it one more bounded wait
  cluster_sync_all();  // no rank leaves while another still reads its shared memory
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
  int early = 0;  // the first cache chunk is loaded before the wait for the previous kernel
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
  r.early = 1;
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
extern "C++" {  // a template inside the C-linkage block
template <int G>
static cudaError_t launch_attention(cudaLaunchConfig_t& cfg, const float* q, const float* k_new, const float* v_new,
                                    float* k_cache, float* v_cache, const int32_t* pos, float* out, int heads,
                                    int kv_heads, int head_dim, int max_len, float scale, const RopeArgs& rope) {
  static std::atomic<uint64_t> attr_set{0};  // per device, per instantiation
  const cudaError_t e =
      set_smem_limit_once(attention_decode_kernel<G>, 2 * kAttnChunk * kAttnMaxDim * (int)sizeof(float), attr_set);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, attention_decode_kernel<G>, q, k_new, v_new, k_cache, v_cache, pos, out, heads,
                            kv_heads, head_dim, max_len, scale, rope.q_w, rope.k_w, rope.cos_t, rope.sin_t, rope.eps,
                            rope.early);
}
}  // extern "C++"

tq4_status attention_impl(const float* q, const float* k_new, const float* v_new, float* k_cache, float* v_cache,
                          const int32_t* pos, float* out, int heads, int kv_heads, int head_dim, int max_len,
                          void* stream, const RopeArgs& rope) {
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !pos || !out || heads <= 0 || kv_heads <= 0 ||
      heads % kv_heads || heads / kv_heads > kAttnMaxGroup || head_dim <= 0 || head_dim > kAttnMaxDim ||
      (head_dim & 3) || max_len <= 0 || kv_heads > 65535 ||
      ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
        reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
        reinterpret_cast<uintptr_t>(rope.q_w) | reinterpret_cast<uintptr_t>(rope.k_w)) & 15)) {
    set_error("tq4_attention_decode: bad arguments (heads a multiple of kv_heads, at most %d query heads per "
              "KV head, head_dim a multiple of 4 and <= %d, q / K / V / norm-weight pointers 16-byte aligned)",
              kAttnMaxGroup, kAttnMaxDim);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int chunks = (max_len + kAttnChunk - 1) / kAttnChunk;
  const int C = std::min(kAttnMaxCluster, chunks);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, kv_heads);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = (size_t)2 * kAttnChunk * head_dim * sizeof(float);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaError_t e;
  switch (heads / kv_heads) {
#define TQ4_ATTN_G(GG)                                                                                      \
  case GG:                                                                                                  \
    e = launch_attention<GG>(cfg, q, k_new, v_new, k_cache, v_cache, pos, out, heads, kv_heads, head_dim,  \
                             max_len, scale, rope);                                                         \
    break;
    TQ4_ATTN_G(1) TQ4_ATTN_G(2) TQ4_ATTN_G(3) TQ4_ATTN_G(4) TQ4_ATTN_G(5) TQ4_ATTN_G(6) TQ4_ATTN_G(7)
    TQ4_ATTN_G(8)
#undef TQ4_ATTN_G
    default:
      set_error("tq4_attention_decode: more than %d query heads per KV head", kAttnMaxGroup);
      return TQ4_ERR_INVALID_ARGUMENT;
  }
  TQ4_CUDA(e);
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
