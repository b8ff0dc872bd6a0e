// Fused unpack + dequantize + GEMV for decode-shaped MatMulNBits calls (M <= 16).
//
// Math (the MatMulNBits clause, quantized.ex:30-46 with dequantize_weight/4 at :234-240):
//   Y[m][n] = sum_k A[m][k] * (q[n][k] - z[n][b(k)]) * s[n][b(k)]
// is evaluated per "segment" (a run of seg = min(block_size, group, 128) elements of one block):
//   Y[m][n] = sum_seg s[n][b] * ( E[m][seg] * P[m][n][seg] - z[n][b] * ZA[m][seg] )
//   P = sum_{k in seg} q[n][k] * a'[m][k]      (tensor cores, exact integer q, f32 accumulate)
//   a' = f16/bf16(A / E),  ZA = E * sum_{k in seg} a'[m][k]
// E is 1 for f16/bf16 activations and an exact power of two for f32 activations (chosen from
// the segment's max |a| so that a' cannot overflow f16). The per-element work is one LOP3 and
// one f16x2/bf16x2 op per two weights; zero points and scales are applied once per segment.
//
// Work split: a CTA of 8 warps owns 16*WN weight rows and a K range of whole 64-byte groups;
// each warp owns 16 rows (mma.sync m16n8k16, weights as the A operand) and every WK-th group of
// the range (WK = 8/WN). Activations, per-segment factors and the CTA's scales / zero points are
// staged once in shared memory; the packed weights stream from HBM with 128-bit non-allocating
// loads, two groups ahead. Warps that share rows reduce through shared memory; CTAs that share
// rows (split-K) reduce through a float workspace, the last CTA of a row tile doing the sum in a
// fixed order (deterministic) and resetting its counter.
#include <map>
#include <memory>
#include <mutex>

#include "internal.cuh"

namespace tq4 {

struct GemvArgs {
  const uint8_t* q;
  int64_t row_bytes;
  const void* scales;  // [n_pad][blocks_pad] in T
  const void* zps;     // same, or null
  int64_t blocks_pad;
  float z_const;
  int st_bf16;         // 2-byte scale storage is bf16 (else f16)
  int K, N, M;
  int bs_log2, seg_log2;
  const void* a;
  const void* bias;
  tq4_dtype bias_t;
  void* y;
  tq4_dtype y_t;
  int64_t ldy;
  int groups;            // groups per row
  int groups_per_split;  // CTA K range in groups
  int wn;                // warps along N: 1, 2, 4 or 8
  int ksplit;
  int64_t n_pad;
  float* ws;
  int* counters;
};

// ---- weight fragments --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t f16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Pair (e0, e1) -> p0 and pair (e2, e3) -> p1 of step j (within its word) of one row's word x,
// as exact integers q in f16x2 (BF = false) or bf16x2 (BF = true).
template <int BITS, bool BF>
__device__ __forceinline__ void weight_pairs(uint32_t x, int j, uint32_t& p0, uint32_t& p1) {
  if constexpr (BITS == 4) {
    const uint32_t src = (j & 1) ? (x >> 8) : x;
    if constexpr (!BF) {
      p0 = f16x2_sub(lop3_and_or(src, 0x000F000Fu, 0x64006400u), 0x64006400u);
      // 1024 + 16 q -> q via q = r/16 - 64 (exact)
      p1 = f16x2_fma(lop3_and_or(src, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD400D400u);
    } else {
      p0 = bf16x2_sub(lop3_and_or(src, 0x000F000Fu, 0x43004300u), 0x43004300u);
      p1 = bf16x2_sub(lop3_and_or(src >> 4, 0x000F000Fu, 0x43004300u), 0x43004300u);
    }
  } else if constexpr (BITS == 2) {
    const int sub = j & 3;
    if constexpr (!BF) {
      const uint32_t src = (sub >= 2) ? (x >> 8) : x;
      const int i0 = 2 * (sub & 1);
      // mask 3 << 2i yields 1024 + 4^i q; scale back by 4^-i and subtract 1024 * 4^-i.
      const uint32_t m0 = 0x00030003u << (2 * i0), m1 = 0x00030003u << (2 * i0 + 2);
      const uint32_t sc0 = (i0 == 0) ? 0x3C003C00u : 0x2C002C00u;  // 1, 1/16
      const uint32_t of0 = (i0 == 0) ? 0xE400E400u : 0xD400D400u;  // -1024, -64
      const uint32_t sc1 = (i0 == 0) ? 0x34003400u : 0x24002400u;  // 1/4, 1/64
      const uint32_t of1 = (i0 == 0) ? 0xDC00DC00u : 0xCC00CC00u;  // -256, -16
      p0 = f16x2_fma(lop3_and_or(src, m0, 0x64006400u), sc0, of0);
      p1 = f16x2_fma(lop3_and_or(src, m1, 0x64006400u), sc1, of1);
    } else {
      const int pos0 = 2 * sub;
      p0 = bf16x2_sub(lop3_and_or(x >> (2 * pos0), 0x00030003u, 0x43004300u), 0x43004300u);
      p1 = bf16x2_sub(lop3_and_or(x >> (2 * pos0 + 2), 0x00030003u, 0x43004300u), 0x43004300u);
    }
  } else {  // 8 bits: the word is one step, bytes e0..e3
    if constexpr (!BF) {
      p0 = f16x2_sub(prmt(x, 0x64646464u, 0x4140u), 0x64006400u);
      p1 = f16x2_sub(prmt(x, 0x64646464u, 0x4342u), 0x64006400u);
    } else {
      const float f0 = __uint_as_float(prmt(x, 0x4B000000u, 0x7540u)) - 8388608.f;
      const float f1 = __uint_as_float(prmt(x, 0x4B000000u, 0x7541u)) - 8388608.f;
      const float f2 = __uint_as_float(prmt(x, 0x4B000000u, 0x7542u)) - 8388608.f;
      const float f3 = __uint_as_float(prmt(x, 0x4B000000u, 0x7543u)) - 8388608.f;
      __nv_bfloat162 h0 = __floats2bfloat162_rn(f0, f1), h1 = __floats2bfloat162_rn(f2, f3);
      p0 = *reinterpret_cast<uint32_t*>(&h0);
      p1 = *reinterpret_cast<uint32_t*>(&h1);
    }
  }
}

template <bool BF>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (!BF) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float scale_to_f32(const void* base, int64_t i, int st_bytes, int bf) {
  if (st_bytes == 4) return static_cast<const float*>(base)[i];
  const uint16_t v = static_cast<const uint16_t*>(base)[i];
  if (bf) return __uint_as_float(((uint32_t)v) << 16);
  return __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int w) {
  return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
}

constexpr int kGemvThreads = 256;
constexpr int kPrefetch = 2;  // groups per load batch (two batches in flight)

template <int BITS, tq4_dtype AT, int ST_BYTES, int MT>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs p) {
  constexpr bool BF = (AT == TQ4_BF16);
  constexpr int G = 512 / BITS;  // elements per 64-byte group
  constexpr int STEPS = G / 16;
  constexpr int STEPS_PER_WORD = 32 / BITS / 4;  // 2 (4-bit), 4 (2-bit), 1 (8-bit)
  constexpr int MP = 8 * MT;
  extern __shared__ __align__(16) uint8_t smem[];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wn = p.wn, wk = 8 / wn;
  const int warp_n = warp % wn, warp_k = warp / wn;
  const int rows_cta = 16 * wn;
  const int64_t cta_row0 = (int64_t)blockIdx.x * rows_cta;
  const int64_t row0 = cta_row0 + warp_n * 16;
  const int split = blockIdx.y;
  const int g_begin = split * p.groups_per_split;
  const int g_end = min(p.groups, g_begin + p.groups_per_split);
  const int kr = (g_end - g_begin) * G;
  const int k0 = g_begin * G;
  const int seg_log2 = p.seg_log2;
  const int seg = 1 << seg_log2;
  const int nseg = kr >> seg_log2;
  const int sk = kr + 16;
  const int b_first = k0 >> p.bs_log2;
  const int nblk = ((k0 + kr - 1) >> p.bs_log2) - b_first + 1;
  const bool has_zp = p.zps != nullptr;

  uint16_t* act = reinterpret_cast<uint16_t*>(smem);
  float* segE = reinterpret_cast<float*>(smem + (size_t)MP * sk * 2);
  float* segZA = segE + MP * nseg;
  float* sc = segZA + MP * nseg;                       // [rows_cta][nblk] as f32
  float* zc = sc + rows_cta * nblk;                    // same (if zero points)

  // -- issue the first weight loads before staging (they overlap the staging latency)
  const uint8_t* rowg = p.q + (row0 + g) * p.row_bytes + t * 16;
  const uint8_t* rowg8 = rowg + 8 * p.row_bytes;
  uint4 xa[kPrefetch], xb[kPrefetch];     // the batch being computed
  uint4 na[kPrefetch], nb[kPrefetch];     // the next batch, in flight
  const int c_first = g_begin + warp_k;
#pragma unroll
  for (int d = 0; d < kPrefetch; ++d) {
    const int c = c_first + d * wk;
    xa[d] = xb[d] = make_uint4(0, 0, 0, 0);
    if (c < g_end) {
      xa[d] = ld_stream(rowg + (int64_t)c * 64);
      xb[d] = ld_stream(rowg8 + (int64_t)c * 64);
    }
  }

  // -- stage the CTA's scales and zero points (as f32)
  for (int i = threadIdx.x; i < rows_cta * nblk; i += kGemvThreads) {
    const int r = i / nblk, bb = i % nblk;
    const int64_t src = (cta_row0 + r) * p.blocks_pad + b_first + bb;
    sc[i] = scale_to_f32(p.scales, src, ST_BYTES, p.st_bf16);
    if (has_zp) zc[i] = scale_to_f32(p.zps, src, ST_BYTES, p.st_bf16);
  }

  // -- stage the activations: a' = A/E in the MMA type, per-segment E and E*sum(a')
  {
    const int vec_per_row = kr / 4;
    const int total_vec = MP * vec_per_row;  // a multiple of 32: whole warps iterate together
    const int L = seg >> 2;                  // lanes per segment (<= 32)
    for (int v = threadIdx.x; v < total_vec; v += kGemvThreads) {
      const int m = v / vec_per_row;
      const int kk = (v % vec_per_row) * 4;
      const int64_t k = (int64_t)k0 + kk;
      float a4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a4[i] = 0.f;
        if (m < p.M && k + i < p.K) a4[i] = load_as_f32(p.a, (int64_t)m * p.K + k + i, AT);
      }
      float e_scale = 1.f, inv = 1.f;
      if constexpr (AT == TQ4_F32) {
        float mx = fmaxf(fmaxf(fabsf(a4[0]), fabsf(a4[1])), fmaxf(fabsf(a4[2]), fabsf(a4[3])));
        for (int off = 1; off < L; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        if (mx > 0.f && mx <= 3.402823466e38f) {
          int ex;
          frexpf(mx, &ex);  // mx = f * 2^ex, f in [0.5, 1)
          const int s = max(-126, min(127, ex - 15));  // mx / 2^s in [2^14, 2^15)
          e_scale = ldexpf(1.f, s);
          inv = ldexpf(1.f, -s);
        }
      }
      uint16_t h[4];
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (BF) {
          const __nv_bfloat16 b = __float2bfloat16_rn(a4[i] * inv);
          h[i] = __bfloat16_as_ushort(b);
          sum += __bfloat162float(b);
        } else {
          const __half b = __float2half_rn(a4[i] * inv);
          h[i] = __half_as_ushort(b);
          sum += __half2float(b);
        }
      }
      for (int off = 1; off < L; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      uint2 packed;
      packed.x = (uint32_t)h[0] | ((uint32_t)h[1] << 16);
      packed.y = (uint32_t)h[2] | ((uint32_t)h[3] << 16);
      *reinterpret_cast<uint2*>(act + m * sk + kk) = packed;
      if ((lane & (L - 1)) == 0) {
        const int s_idx = kk >> seg_log2;
        segE[m * nseg + s_idx] = e_scale;
        segZA[m * nseg + s_idx] = e_scale * sum;
      }
    }
  }
  __syncthreads();

  // -- main loop: this warp's groups c = c_first + i*wk, batches of kPrefetch, two in flight
  float acc[MT][4];
  float blk[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][i] = blk[mt][i] = 0.f;

  const int rl_g = warp_n * 16 + g;  // row of this thread's weights within the CTA
  for (int cb = c_first; cb < g_end; cb += kPrefetch * wk) {
    // issue the next batch before computing this one
    const int cn = cb + kPrefetch * wk;
#pragma unroll
    for (int d = 0; d < kPrefetch; ++d) {
      const int c = cn + d * wk;
      na[d] = nb[d] = make_uint4(0, 0, 0, 0);
      if (c < g_end) {
        na[d] = ld_stream(rowg + (int64_t)c * 64);
        nb[d] = ld_stream(rowg8 + (int64_t)c * 64);
      }
    }
#pragma unroll
    for (int d = 0; d < kPrefetch; ++d) {
      const int c = cb + d * wk;
      if (c >= g_end) break;
      const int kc = (c - g_begin) * G;  // group's first element within the CTA range
#pragma unroll
      for (int j = 0; j < STEPS; ++j) {
        const int w = j / STEPS_PER_WORD;
        uint32_t a0, a1, a2, a3;
        weight_pairs<BITS, BF>(word_of(xa[d], w), j, a0, a2);
        weight_pairs<BITS, BF>(word_of(xb[d], w), j, a1, a3);
        const int kk = kc + 16 * j + 4 * t;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint2 bv = *reinterpret_cast<const uint2*>(act + (mt * 8 + g) * sk + kk);
          mma16816<BF>(blk[mt], a0, a1, a2, a3, bv.x, bv.y);
        }
        if ((((j + 1) * 16) & (seg - 1)) == 0) {  // end of a segment
          const int s_idx = (kc + (j + 1) * 16 - seg) >> seg_log2;
          const int bb = ((k0 + s_idx * seg) >> p.bs_log2) - b_first;
          const float s_g = sc[rl_g * nblk + bb], s_g8 = sc[(rl_g + 8) * nblk + bb];
          const float z_g = has_zp ? zc[rl_g * nblk + bb] : p.z_const;
          const float z_g8 = has_zp ? zc[(rl_g + 8) * nblk + bb] : p.z_const;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int m0 = mt * 8 + 2 * t;
            const float E0 = segE[m0 * nseg + s_idx], ZA0 = segZA[m0 * nseg + s_idx];
            const float E1 = segE[(m0 + 1) * nseg + s_idx], ZA1 = segZA[(m0 + 1) * nseg + s_idx];
            acc[mt][0] = fmaf(s_g, fmaf(E0, blk[mt][0], -z_g * ZA0), acc[mt][0]);
            acc[mt][1] = fmaf(s_g, fmaf(E1, blk[mt][1], -z_g * ZA1), acc[mt][1]);
            acc[mt][2] = fmaf(s_g8, fmaf(E0, blk[mt][2], -z_g8 * ZA0), acc[mt][2]);
            acc[mt][3] = fmaf(s_g8, fmaf(E1, blk[mt][3], -z_g8 * ZA1), acc[mt][3]);
#pragma unroll
            for (int i = 0; i < 4; ++i) blk[mt][i] = 0.f;
          }
        }
      }
    }
#pragma unroll
    for (int d = 0; d < kPrefetch; ++d) {
      xa[d] = na[d];
      xb[d] = nb[d];
    }
  }

  // -- reduce the warps that share rows (fixed order)
  __syncthreads();  // all warps are done with the staged data
  float* red = reinterpret_cast<float*>(smem);  // [8 warps][32 lanes][MT*4]
  if (wk > 1) {
    if (warp_k > 0) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[(warp * 32 + lane) * (MT * 4) + mt * 4 + i] = acc[mt][i];
    }
    __syncthreads();
    if (warp_k == 0) {
      for (int kk = 1; kk < wk; ++kk) {
        const int src = (kk * wn + warp_n) * 32 + lane;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[mt][i] += red[src * (MT * 4) + mt * 4 + i];
      }
    }
  }

  const int64_t n_g = row0 + g, n_g8 = row0 + g + 8;
  if (p.ksplit == 1) {
    if (warp_k == 0) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int m = mt * 8 + 2 * t + (i & 1);
          const int64_t n = (i < 2) ? n_g : n_g8;
          if (m < p.M && n < p.N) {
            float v = acc[mt][i];
            if (p.bias) v = round_to(v, p.y_t) + load_as_f32(p.bias, n, p.bias_t);
            store_from_f32(p.y, (int64_t)m * p.ldy + n, p.y_t, v);
          }
        }
      }
    }
    return;
  }

  // -- split-K: write this CTA's partial, the last CTA of the row tile sums them in order
  if (warp_k == 0) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = mt * 8 + 2 * t + (i & 1);
        const int64_t n = (i < 2) ? n_g : n_g8;
        if (m < p.M) p.ws[((int64_t)split * p.M + m) * p.n_pad + n] = acc[mt][i];
      }
  }
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&p.counters[blockIdx.x], 1);
    s_last = (prev == p.ksplit - 1);
    if (prev >= p.ksplit) report(kDevTimeoutSplitK);  // a counter left non-zero by a failed call
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int outputs = rows_cta * p.M;
  for (int i = threadIdx.x; i < outputs; i += kGemvThreads) {
    const int m = i / rows_cta;
    const int64_t n = cta_row0 + (i % rows_cta);
    if (n >= p.N) continue;
    float v = 0.f;
    for (int s = 0; s < p.ksplit; ++s) v += __ldcg(&p.ws[((int64_t)s * p.M + m) * p.n_pad + n]);
    if (p.bias) v = round_to(v, p.y_t) + load_as_f32(p.bias, n, p.bias_t);
    store_from_f32(p.y, (int64_t)m * p.ldy + n, p.y_t, v);
  }
  if (threadIdx.x == 0) p.counters[blockIdx.x] = 0;
}

// ---- host side --------------------------------------------------------------------------------
struct GemvPlan {
  int wn, ksplit, groups_per_split, mt, ctas_n;
  size_t smem;
};

static size_t gemv_smem(int mt, int kr, int seg, int rows_cta, int nblk, bool zp) {
  const int mp = 8 * mt;
  size_t bytes = (size_t)mp * (kr + 16) * 2 + (size_t)2 * mp * (kr / seg) * 4 +
                 (size_t)rows_cta * nblk * 4 * (zp ? 2 : 1);
  const size_t red = (size_t)8 * 32 * mt * 4 * 4;
  return std::max(bytes, red);
}

static GemvPlan plan_gemv(const Weight& w, int64_t m) {
  GemvPlan pl{};
  const int bits = w.desc.bits;
  const int G = 512 / bits;
  const int seg = std::min<int>(std::min(w.desc.block_size, G), 128);
  pl.mt = m <= 8 ? 1 : 2;
  const int sms = w.num_sms;
  const int target = 2 * sms;
  const int64_t groups = w.groups;
  pl.wn = 1;
  for (int wn = 8; wn >= 1; wn >>= 1) {
    const int64_t ctas = (w.n_pad + 16 * wn - 1) / (16 * wn);
    if (ctas >= target || wn == 1) {
      pl.wn = wn;
      break;
    }
  }
  pl.ctas_n = (int)((w.n_pad + 16 * pl.wn - 1) / (16 * pl.wn));
  const int wk = 8 / pl.wn;
  int ksplit = 1;
  if (pl.ctas_n < target) ksplit = (int)std::min<int64_t>((target + pl.ctas_n - 1) / pl.ctas_n,
                                                         std::max<int64_t>(1, groups / wk));
  // shared-memory budget: shrink the per-CTA K range until the staging fits
  const size_t budget = 100 * 1024;
  const bool zp = w.zps.ptr != nullptr;
  const int rows_cta = 16 * pl.wn;
  for (;;) {
    const int gps = (int)((groups + ksplit - 1) / ksplit);
    const int kr = gps * G;
    const int nblk = (kr + w.desc.block_size - 1) / w.desc.block_size + 1;
    const size_t smem = gemv_smem(pl.mt, kr, seg, rows_cta, nblk, zp);
    if (smem <= budget || gps == 1) {
      pl.groups_per_split = gps;
      pl.smem = smem;
      break;
    }
    ++ksplit;
  }
  // every split must own at least one group
  pl.ksplit = (int)((groups + pl.groups_per_split - 1) / pl.groups_per_split);
  return pl;
}

template <int BITS, tq4_dtype AT, int ST, int MT>
static cudaError_t launch_gemv_t(const GemvArgs& args, dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = gemv_kernel<BITS, AT, ST, MT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kGemvThreads, smem, st>>>(args);
  return cudaGetLastError();
}

template <int BITS, tq4_dtype AT>
static cudaError_t launch_gemv_st(const GemvArgs& args, int st_bytes, int mt, dim3 grid, size_t smem,
                                  cudaStream_t st) {
  if (st_bytes == 4) {
    return mt == 1 ? launch_gemv_t<BITS, AT, 4, 1>(args, grid, smem, st)
                   : launch_gemv_t<BITS, AT, 4, 2>(args, grid, smem, st);
  }
  return mt == 1 ? launch_gemv_t<BITS, AT, 2, 1>(args, grid, smem, st)
                 : launch_gemv_t<BITS, AT, 2, 2>(args, grid, smem, st);
}

template <int BITS>
static cudaError_t launch_gemv_bits(const GemvArgs& args, tq4_dtype a_t, int st_bytes, int mt,
                                    dim3 grid, size_t smem, cudaStream_t st) {
  switch (a_t) {
    case TQ4_F16: return launch_gemv_st<BITS, TQ4_F16>(args, st_bytes, mt, grid, smem, st);
    case TQ4_BF16: return launch_gemv_st<BITS, TQ4_BF16>(args, st_bytes, mt, grid, smem, st);
    default: return launch_gemv_st<BITS, TQ4_F32>(args, st_bytes, mt, grid, smem, st);
  }
}

// Per-stream split-K workspaces of a handle: calls on different streams may overlap on the GPU,
// so each stream gets its own partial-sum buffer and counters.
struct Workspace {
  DeviceBuffer ws, counters;
};
struct WorkspaceMap {
  std::mutex mu;
  std::map<cudaStream_t, std::unique_ptr<Workspace>> by_stream;
};

static WorkspaceMap& workspaces(const Weight& w) {
  static std::mutex create_mu;
  std::lock_guard<std::mutex> lock(create_mu);
  Weight& mw = const_cast<Weight&>(w);
  if (!mw.ws_mutex) mw.ws_mutex = new WorkspaceMap();
  return *static_cast<WorkspaceMap*>(mw.ws_mutex);
}

void free_workspaces(Weight& w) {
  delete static_cast<WorkspaceMap*>(w.ws_mutex);
  w.ws_mutex = nullptr;
}

tq4_status gemv_workspace(const Weight& w, cudaStream_t st, int64_t ws_bytes, int64_t ctr_count,
                          float** ws, int** counters) {
  WorkspaceMap& map = workspaces(w);
  std::lock_guard<std::mutex> lock(map.mu);
  auto& slot = map.by_stream[st];
  if (!slot) slot.reset(new Workspace());
  if (slot->ws.bytes < ws_bytes) TQ4_TRY(slot->ws.alloc(ws_bytes));
  if (slot->counters.bytes < ctr_count * 4) {
    TQ4_TRY(slot->counters.alloc(ctr_count * 4));
    TQ4_CUDA(cudaMemsetAsync(slot->counters.ptr, 0, ctr_count * 4, st));
  }
  *ws = static_cast<float*>(slot->ws.ptr);
  *counters = static_cast<int*>(slot->counters.ptr);
  return TQ4_OK;
}

tq4_status run_gemv_with(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                         tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st, float* ws,
                         int* counters, int64_t ws_capacity_floats, int64_t ctr_capacity) {
  const GemvPlan pl = plan_gemv(w, m);
  GemvArgs args{};
  args.q = static_cast<const uint8_t*>(w.q.ptr);
  args.row_bytes = w.row_bytes;
  args.scales = w.scales.ptr;
  args.zps = w.zps.ptr;
  args.blocks_pad = w.blocks_pad;
  args.z_const = w.z_const;
  args.st_bf16 = w.desc.dequant_dtype == TQ4_BF16;
  args.K = (int)w.desc.K;
  args.N = (int)w.desc.N;
  args.M = (int)m;
  args.bs_log2 = w.bs_log2;
  const int G = 512 / w.desc.bits;
  const int seg = std::min<int>(std::min(w.desc.block_size, G), 128);
  int seg_log2 = 0;
  while ((1 << seg_log2) < seg) ++seg_log2;
  args.seg_log2 = seg_log2;
  args.a = a;
  args.bias = bias;
  args.bias_t = bias_t;
  args.y = y;
  args.y_t = y_t;
  args.ldy = ldy;
  args.groups = (int)w.groups;
  args.groups_per_split = pl.groups_per_split;
  args.wn = pl.wn;
  args.ksplit = pl.ksplit;
  args.n_pad = w.n_pad;
  if (pl.ksplit > 1) {
    const int64_t need = (int64_t)pl.ksplit * m * w.n_pad;
    if (ws == nullptr || need > ws_capacity_floats || pl.ctas_n > ctr_capacity) {
      set_error("split-K workspace too small: need %lld floats and %d counters",
                (long long)need, pl.ctas_n);
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    args.ws = ws;
    args.counters = counters;
  }
  const dim3 grid(pl.ctas_n, pl.ksplit);
  const int st_bytes = w.desc.dequant_dtype == TQ4_F32 ? 4 : 2;
  cudaError_t e;
  if (w.desc.bits == 4) e = launch_gemv_bits<4>(args, a_t, st_bytes, pl.mt, grid, pl.smem, st);
  else if (w.desc.bits == 2) e = launch_gemv_bits<2>(args, a_t, st_bytes, pl.mt, grid, pl.smem, st);
  else e = launch_gemv_bits<8>(args, a_t, st_bytes, pl.mt, grid, pl.smem, st);
  if (e != cudaSuccess) {
    set_error("GEMV launch failed: %s", cudaGetErrorString(e));
    return TQ4_ERR_CUDA;
  }
  return TQ4_OK;
}

int64_t gemv_workspace_floats(const Weight& w, int64_t m) {
  const GemvPlan pl = plan_gemv(w, m);
  return pl.ksplit > 1 ? (int64_t)pl.ksplit * m * w.n_pad : 0;
}

int64_t gemv_counter_count(const Weight& w, int64_t m) { return plan_gemv(w, m).ctas_n; }

tq4_status run_gemv(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                    tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  float* ws = nullptr;
  int* ctr = nullptr;
  const int64_t need = gemv_workspace_floats(w, m);
  const int64_t nctr = gemv_counter_count(w, m);
  if (need > 0) TQ4_TRY(gemv_workspace(w, st, need * 4, nctr, &ws, &ctr));
  return run_gemv_with(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st, ws, ctr, need, nctr);
}

}  // namespace tq4
