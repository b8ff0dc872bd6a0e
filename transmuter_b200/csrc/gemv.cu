// Fused unpack + dequantize + GEMV for decode-shaped MatMulNBits calls (M <= 16).
//
// Math (the MatMulNBits clause, quantized.ex:30-46 with dequantize_weight/4 at :234-240):
//   Y[m][n] = sum_k A[m][k] * (q[n][k] - z[n][b(k)]) * s[n][b(k)]
// is evaluated per "segment" (a run of seg = min(block_size, group, 128) weights of one block).
// The weights enter the tensor cores as magic-number floats O + q*c(k)^-1 straight out of one
// LOP3 (O = 1024 for f16, 128 for bf16; c(k) is 1/16, 1/4, ... for the nibbles the mask leaves
// shifted, and the staged activation at k is multiplied by c(k) to match). With the staged
// activations v(k) = RN(A[m][k] / E * c(k)) (E an exact power of two per segment chosen so that
// v cannot overflow f16),
//   P[m][n][seg] = sum_{k in seg} (O + q/c(k)) v(k)            (mma.sync, f32 accumulate)
//   Y[m][n]     += s[n][b] * ( E*P - E*O*SV - z[n][b] * E*SA ),  SV = sum v, SA = sum v/c
// so zero points, scales and the magic offset cost a few FMAs per segment and each pair of
// weights costs one LOP3 (plus one shift per 32-bit word).
//
// Work split: a tile is 16*WN weight rows x a K range of whole 64-byte groups; persistent CTAs
// of 8 warps walk the tiles. Each warp owns 16 rows of the tile (mma.sync m16n8k16, weights as
// the A operand) and every WK-th group of the range (WK = 8/WN). Activations and per-segment
// factors are staged in shared memory once per K range; each tile's scales / zero points arrive
// by cp.async (block-major, so each block's rows are one contiguous run) while its first weights
// are in flight; the packed weights stream from HBM with 128-bit non-allocating loads, two
// groups ahead. Warps that share rows reduce through shared memory; tiles that share rows
// (split-K) reduce through a float workspace, the last CTA of a row tile doing the sum in a
// fixed order (deterministic) and resetting its counter.
#include <map>
#include <memory>
#include <mutex>

#include "internal.cuh"

namespace tq4 {

struct GemvArgs {
  const uint8_t* q;
  int64_t row_bytes;
  const void* scales;  // [blocks_pad][n_pad] in T
  const void* zps;     // same, or null
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
  int ctas_n;            // row tiles; the persistent grid walks ctas_n * ksplit tiles
  int64_t n_pad;
  float* ws;
  int* counters;
};

// ---- weight fragments --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Magic-number weights of step j (within its word) of one row's word x: p0 holds the pair
// (e0, e1), p1 the pair (e2, e3), each as O + q/c in f16x2 (BF = false) or bf16x2 (BF = true).
// PRECISE (f32 activations) keeps the offset small against the weights: every 4-bit pair comes
// out as 1024 + 16 q (one more shift per word) and 2-bit weights come out as exact q, so the
// f32 accumulator never carries terms much larger than the result it is building.
template <int BITS, bool BF, bool PRECISE>
__device__ __forceinline__ void weight_pairs(uint32_t x, int j, uint32_t& p0, uint32_t& p1) {
  if constexpr (BITS == 4) {
    const uint32_t src = (j & 1) ? (x >> 8) : x;
    if constexpr (!BF && PRECISE) {
      p0 = lop3_and_or((j & 1) ? (x >> 4) : (x << 4), 0x00F000F0u, 0x64006400u);  // 1024 + 16 q
      p1 = lop3_and_or(src, 0x00F000F0u, 0x64006400u);                           // 1024 + 16 q
    } else if constexpr (!BF) {
      p0 = lop3_and_or(src, 0x000F000Fu, 0x64006400u);  // 1024 + q
      p1 = lop3_and_or(src, 0x00F000F0u, 0x64006400u);  // 1024 + 16 q
    } else {
      p0 = lop3_and_or(src, 0x000F000Fu, 0x43004300u);       // 128 + q
      p1 = lop3_and_or(src >> 4, 0x000F000Fu, 0x43004300u);  // 128 + q
    }
  } else if constexpr (BITS == 2) {
    const int sub = j & 3;
    if constexpr (!BF) {
      const uint32_t src = (sub >= 2) ? (x >> 8) : x;
      const int i0 = 2 * (sub & 1);
      p0 = lop3_and_or(src, 0x00030003u << (2 * i0), 0x64006400u);      // 1024 + 4^i0 q
      p1 = lop3_and_or(src, 0x00030003u << (2 * i0 + 2), 0x64006400u);  // 1024 + 4^(i0+1) q
      if constexpr (PRECISE) {  // exact q: r * 4^-i - 1024 * 4^-i
        const uint32_t sc0 = (i0 == 0) ? 0x3C003C00u : 0x2C002C00u;  // 1, 1/16
        const uint32_t of0 = (i0 == 0) ? 0xE400E400u : 0xD400D400u;  // -1024, -64
        const uint32_t sc1 = (i0 == 0) ? 0x34003400u : 0x24002400u;  // 1/4, 1/64
        const uint32_t of1 = (i0 == 0) ? 0xDC00DC00u : 0xCC00CC00u;  // -256, -16
        asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(p0) : "r"(sc0), "r"(of0));
        asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(p1) : "r"(sc1), "r"(of1));
      }
    } else {
      const int pos0 = 2 * sub;
      p0 = lop3_and_or(x >> (2 * pos0), 0x00030003u, 0x43004300u);
      p1 = lop3_and_or(x >> (2 * pos0 + 2), 0x00030003u, 0x43004300u);
    }
  } else {  // 8 bits: the word is one step, bytes e0..e3
    if constexpr (!BF) {
      p0 = prmt(x, 0x64646464u, 0x4140u);  // 1024 + q
      p1 = prmt(x, 0x64646464u, 0x4342u);
    } else {  // exact q through f32 (bf16 cannot hold 128 + q for q >= 128)
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

// The offset O of the magic-number weights and the activation factor c(k) that matches the
// weight at position k (k is the position within the 64-byte group's elements).
template <int BITS, bool BF, bool PRECISE>
__device__ __forceinline__ float magic_offset() {
  if constexpr (BITS == 8 && BF) return 0.f;
  if constexpr (BITS == 2 && !BF && PRECISE) return 0.f;
  return BF ? 128.f : 1024.f;
}
template <int BITS, bool BF, bool PRECISE>
__device__ __forceinline__ float act_factor(int k) {
  if constexpr (BF) return 1.f;
  if constexpr (BITS == 4 && PRECISE) return 0.0625f;
  if constexpr (BITS == 4) return (k & 2) ? 0.0625f : 1.f;
  if constexpr (BITS == 2 && PRECISE) return 1.f;
  if constexpr (BITS == 2) {
    const int i = 2 * ((k >> 4) & 1) + ((k >> 1) & 1);
    return i == 0 ? 1.f : (i == 1 ? 0.25f : (i == 2 ? 0.0625f : 0.015625f));
  }
  return 1.f;
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

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Four consecutive activations A[m][k..k+3] as f32 (zeros past K). `vec` when a 4-wide load is
// aligned (K % 4 == 0).
template <tq4_dtype AT>
__device__ __forceinline__ void load_act4(const void* a, int64_t m, int64_t k, int K, bool vec,
                                          float (&out)[4]) {
  const int64_t i = m * K + k;
  if (vec && k + 3 < K) {
    if constexpr (AT == TQ4_F32) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a) + i));
      out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
    } else {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(a) + i));
      const uint32_t h[4] = {v.x & 0xFFFF, v.x >> 16, v.y & 0xFFFF, v.y >> 16};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        out[e] = (AT == TQ4_BF16) ? __uint_as_float(h[e] << 16) : __half2float(__ushort_as_half((uint16_t)h[e]));
    }
    return;
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) out[e] = (k + e < K) ? load_as_f32(a, i + e, AT) : 0.f;
}

// Stages A[0:M][k0 : k0+kr] into shared memory as v(k) = RN(A / E * c(k)) in the MMA type, with
// the per-segment factors {E, E*O*SV - (no zero points ? z*E*SA : 0), E*SA} as float4 [seg][m].
// Rows >= M are left as they are: their outputs are never stored, and an MMA output element
// depends only on its own activation row.
template <int BITS, tq4_dtype AT>
__device__ __forceinline__ void stage_activations(const GemvArgs& p, int k0, int kr, int sk, int mp,
                                                  uint16_t* act, float4* segf) {
  constexpr bool BF = (AT == TQ4_BF16);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vec_per_row = kr / 4;
  const int total = p.M * vec_per_row;
  const int total_pad = (total + 31) & ~31;  // whole warps take part in the shuffles
  const int L = (1 << p.seg_log2) >> 2;      // lanes per segment (<= 32)
  const bool vec = (p.K & 3) == 0;
  constexpr bool PRECISE = (AT == TQ4_F32);
  const float O = magic_offset<BITS, BF, PRECISE>();
  const bool fold_z = p.zps == nullptr;
  for (int base = 0; base < total_pad; base += 4 * kGemvThreads) {
    float a4[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {  // issue all loads first
      const int v = base + u * kGemvThreads + threadIdx.x;
      if (v < total) {
        load_act4<AT>(p.a, v / vec_per_row, (int64_t)k0 + (v % vec_per_row) * 4, p.K, vec, a4[u]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) a4[u][e] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (base + u * kGemvThreads + warp * 32 >= total_pad) continue;  // warp-uniform
      const int v = base + u * kGemvThreads + threadIdx.x;
      const int m = v / vec_per_row, kk = (v % vec_per_row) * 4;
      float mx = fmaxf(fmaxf(fabsf(a4[u][0]), fabsf(a4[u][1])), fmaxf(fabsf(a4[u][2]), fabsf(a4[u][3])));
      for (int off = 1; off < L; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      float e_scale = 1.f, inv = 1.f;
      if (mx > 0.f && mx <= 3.402823466e38f) {
        int ex;
        frexpf(mx, &ex);                             // mx = f * 2^ex, f in [0.5, 1)
        const int s = max(-126, min(127, ex - 15));  // mx / 2^s in [2^14, 2^15)
        e_scale = ldexpf(1.f, s);
        inv = ldexpf(1.f, -s);
      }
      uint16_t h[4];
      float sv = 0.f, sa = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float c = act_factor<BITS, BF, PRECISE>(kk + e);  // kk: a multiple of 4
        float val;
        if constexpr (BF) {
          const __nv_bfloat16 b = __float2bfloat16_rn(a4[u][e] * inv * c);
          h[e] = __bfloat16_as_ushort(b);
          val = __bfloat162float(b);
        } else {
          const __half b = __float2half_rn(a4[u][e] * inv * c);
          h[e] = __half_as_ushort(b);
          val = __half2float(b);
        }
        sv += val;
        sa += val / c;  // exact: c is a power of two
      }
      for (int off = 1; off < L; off <<= 1) {
        sv += __shfl_xor_sync(0xffffffffu, sv, off);
        sa += __shfl_xor_sync(0xffffffffu, sa, off);
      }
      if (v < total) {
        uint2 packed;
        packed.x = (uint32_t)h[0] | ((uint32_t)h[1] << 16);
        packed.y = (uint32_t)h[2] | ((uint32_t)h[3] << 16);
        *reinterpret_cast<uint2*>(act + m * sk + kk) = packed;
        if ((lane & (L - 1)) == 0) {
          const int s_idx = kk >> p.seg_log2;
          const float za = e_scale * sa;
          const float x = e_scale * O * sv + (fold_z ? p.z_const * za : 0.f);
          segf[s_idx * mp + m] = make_float4(e_scale, x, za, 0.f);
        }
      }
    }
  }
}

// Shared-memory plan of one CTA (identical on host and device).
struct GemvSmem {
  int sk, nseg, nblk_max;
  int act_off, seg_off, sc_off, zc_off, red_off, total;
};

__host__ __device__ inline GemvSmem gemv_smem_plan(int mt, int kr_max, int seg, int bs, int rows_cta,
                                                   int st_bytes, bool zp) {
  GemvSmem s{};
  const int mp = 8 * mt;
  s.sk = kr_max + 16;
  s.nseg = kr_max / seg;
  s.nblk_max = (kr_max + bs - 1) / bs + 1;
  s.act_off = 0;
  s.seg_off = (s.act_off + mp * s.sk * 2 + 15) / 16 * 16;
  s.sc_off = s.seg_off + s.nseg * mp * 16;
  s.zc_off = s.sc_off + (s.nblk_max * rows_cta * st_bytes + 15) / 16 * 16;
  s.red_off = s.zc_off + (zp ? (s.nblk_max * rows_cta * st_bytes + 15) / 16 * 16 : 0);
  s.total = s.red_off + 8 * 32 * mt * 4 * 4;
  return s;
}

template <int BITS, tq4_dtype AT, int ST_BYTES, int MT>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvArgs p) {
  constexpr bool BF = (AT == TQ4_BF16);
  constexpr int G = 512 / BITS;  // elements per 64-byte group
  constexpr int STEPS = G / 16;
  constexpr int STEPS_PER_WORD = 32 / BITS / 4;  // 2 (4-bit), 4 (2-bit), 1 (8-bit)
  constexpr int MP = 8 * MT;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wn = p.wn, wk = 8 / wn;
  const int warp_n = warp % wn, warp_k = warp / wn;
  const int rows_cta = 16 * wn;
  const int seg_log2 = p.seg_log2;
  const int seg = 1 << seg_log2;
  const bool has_zp = p.zps != nullptr;
  const GemvSmem L = gemv_smem_plan(MT, p.groups_per_split * G, seg, 1 << p.bs_log2, rows_cta,
                                    ST_BYTES, has_zp);
  uint16_t* act = reinterpret_cast<uint16_t*>(smem + L.act_off);
  float4* segf = reinterpret_cast<float4*>(smem + L.seg_off);
  uint8_t* sc = smem + L.sc_off;
  uint8_t* zc = smem + L.zc_off;
  float* red = reinterpret_cast<float*>(smem + L.red_off);
  const int sk = L.sk;

  const int tiles = p.ctas_n * p.ksplit;
  int staged_split = -1;
  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int split = tile / p.ctas_n, rt = tile % p.ctas_n;
    const int64_t cta_row0 = (int64_t)rt * rows_cta;
    const int64_t row0 = cta_row0 + warp_n * 16;
    const int g_begin = split * p.groups_per_split;
    const int g_end = min(p.groups, g_begin + p.groups_per_split);
    const int kr = (g_end - g_begin) * G;
    const int k0 = g_begin * G;
    const int b_first = k0 >> p.bs_log2;
    const int nblk = ((k0 + kr - 1) >> p.bs_log2) - b_first + 1;

    // -- scales / zero points of this tile: per block, the tile's rows are one contiguous run
    const int c16 = rows_cta * ST_BYTES / 16;  // 16-byte chunks per block
    for (int i = threadIdx.x; i < nblk * c16; i += kGemvThreads) {
      const int bb = i / c16, c = i % c16;
      const int64_t src = ((int64_t)(b_first + bb) * p.n_pad + cta_row0) * ST_BYTES + c * 16;
      cp_async16(sc + (bb * rows_cta) * ST_BYTES + c * 16, static_cast<const uint8_t*>(p.scales) + src);
      if (has_zp) cp_async16(zc + (bb * rows_cta) * ST_BYTES + c * 16, static_cast<const uint8_t*>(p.zps) + src);
    }

    // -- the first weight batch
    const uint8_t* rowg = p.q + (row0 + g) * p.row_bytes + t * 16;
    const uint8_t* rowg8 = rowg + 8 * p.row_bytes;
    uint4 xa[kPrefetch], xb[kPrefetch];  // the batch being computed
    uint4 na[kPrefetch], nb[kPrefetch];  // the next batch, in flight
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

    // -- activations, once per K range
    if (split != staged_split) {
      stage_activations<BITS, AT>(p, k0, kr, sk, MP, act, segf);
      staged_split = split;
    }
    cp_async_wait_all();
    __syncthreads();

    // -- main loop over this warp's groups
    float acc[MT][4], blk[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][i] = blk[mt][i] = 0.f;
    const int rl_g = warp_n * 16 + g;

    for (int cb = c_first; cb < g_end; cb += kPrefetch * wk) {
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
        const int kc = (c - g_begin) * G;
#pragma unroll
        for (int j = 0; j < STEPS; ++j) {
          const int w = j / STEPS_PER_WORD;
          uint32_t a0, a1, a2, a3;
          weight_pairs<BITS, BF, AT == TQ4_F32>(word_of(xa[d], w), j, a0, a2);
          weight_pairs<BITS, BF, AT == TQ4_F32>(word_of(xb[d], w), j, a1, a3);
          const int kk = kc + 16 * j + 4 * t;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint2 bv = *reinterpret_cast<const uint2*>(act + (mt * 8 + g) * sk + kk);
            mma16816<BF>(blk[mt], a0, a1, a2, a3, bv.x, bv.y);
          }
          if ((((j + 1) * 16) & (seg - 1)) == 0) {  // end of a segment
            const int s_idx = (kc + (j + 1) * 16 - seg) >> seg_log2;
            const int bb = ((k0 + s_idx * seg) >> p.bs_log2) - b_first;
            const float s_g = scale_to_f32(sc, bb * rows_cta + rl_g, ST_BYTES, p.st_bf16);
            const float s_g8 = scale_to_f32(sc, bb * rows_cta + rl_g + 8, ST_BYTES, p.st_bf16);
            const float z_g = has_zp ? scale_to_f32(zc, bb * rows_cta + rl_g, ST_BYTES, p.st_bf16) : 0.f;
            const float z_g8 = has_zp ? scale_to_f32(zc, bb * rows_cta + rl_g + 8, ST_BYTES, p.st_bf16) : 0.f;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const int m0 = mt * 8 + 2 * t;
              const float4 F0 = segf[s_idx * MP + m0], F1 = segf[s_idx * MP + m0 + 1];
              // s * (E*P - X - z*ZA); without zero points X already holds z_const*ZA
              acc[mt][0] = fmaf(s_g, fmaf(-z_g, F0.z, fmaf(F0.x, blk[mt][0], -F0.y)), acc[mt][0]);
              acc[mt][1] = fmaf(s_g, fmaf(-z_g, F1.z, fmaf(F1.x, blk[mt][1], -F1.y)), acc[mt][1]);
              acc[mt][2] = fmaf(s_g8, fmaf(-z_g8, F0.z, fmaf(F0.x, blk[mt][2], -F0.y)), acc[mt][2]);
              acc[mt][3] = fmaf(s_g8, fmaf(-z_g8, F1.z, fmaf(F1.x, blk[mt][3], -F1.y)), acc[mt][3]);
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
    } else {
      // split-K: write this tile's partial; the last CTA of the row tile sums them in order
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
      if (threadIdx.x == 0) {
        const int prev = atomicAdd(&p.counters[rt], 1);
        s_last = (prev == p.ksplit - 1);
        if (prev >= p.ksplit) report(kDevTimeoutSplitK);  // a counter left non-zero earlier
      }
      __syncthreads();
      if (s_last) {
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
        if (threadIdx.x == 0) p.counters[rt] = 0;
      }
    }
    __syncthreads();  // the tile's shared data (scales, reduction) is free again
  }
}

// ---- host side --------------------------------------------------------------------------------
struct GemvPlan {
  int wn, ksplit, groups_per_split, mt, ctas_n;
  size_t smem;
};

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
  const size_t budget = 100 * 1024;
  const bool zp = w.zps.ptr != nullptr;
  const int st_bytes = w.desc.dequant_dtype == TQ4_F32 ? 4 : 2;
  const int rows_cta = 16 * pl.wn;
  for (;;) {
    const int gps = (int)((groups + ksplit - 1) / ksplit);
    const GemvSmem s = gemv_smem_plan(pl.mt, gps * G, seg, w.desc.block_size, rows_cta, st_bytes, zp);
    if ((size_t)s.total <= budget || gps == 1) {
      pl.groups_per_split = gps;
      pl.smem = s.total;
      break;
    }
    ++ksplit;
  }
  pl.ksplit = (int)((groups + pl.groups_per_split - 1) / pl.groups_per_split);
  return pl;
}

template <int BITS, tq4_dtype AT, int ST, int MT>
static cudaError_t launch_gemv_t(const GemvArgs& args, int tiles, int sms, size_t smem, cudaStream_t st) {
  auto kern = gemv_kernel<BITS, AT, ST, MT>;
  // attribute and occupancy once per instantiation (the shared-memory budget is fixed)
  static int per_sm = 0;
  if (per_sm == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024 + 1024);
    if (e != cudaSuccess) return e;
    int n = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kGemvThreads, 100 * 1024);
    if (e != cudaSuccess) return e;
    per_sm = std::max(1, n);
  }
  const int grid = std::min(tiles, per_sm * sms);
  kern<<<grid, kGemvThreads, smem, st>>>(args);
  return cudaGetLastError();
}

template <int BITS, tq4_dtype AT>
static cudaError_t launch_gemv_st(const GemvArgs& args, int st_bytes, int mt, int tiles, int sms,
                                  size_t smem, cudaStream_t st) {
  if (st_bytes == 4) {
    return mt == 1 ? launch_gemv_t<BITS, AT, 4, 1>(args, tiles, sms, smem, st)
                   : launch_gemv_t<BITS, AT, 4, 2>(args, tiles, sms, smem, st);
  }
  return mt == 1 ? launch_gemv_t<BITS, AT, 2, 1>(args, tiles, sms, smem, st)
                 : launch_gemv_t<BITS, AT, 2, 2>(args, tiles, sms, smem, st);
}

template <int BITS>
static cudaError_t launch_gemv_bits(const GemvArgs& args, tq4_dtype a_t, int st_bytes, int mt,
                                    int tiles, int sms, size_t smem, cudaStream_t st) {
  switch (a_t) {
    case TQ4_F16: return launch_gemv_st<BITS, TQ4_F16>(args, st_bytes, mt, tiles, sms, smem, st);
    case TQ4_BF16: return launch_gemv_st<BITS, TQ4_BF16>(args, st_bytes, mt, tiles, sms, smem, st);
    default: return launch_gemv_st<BITS, TQ4_F32>(args, st_bytes, mt, tiles, sms, smem, st);
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

static std::mutex g_ws_create_mu;

static WorkspaceMap& workspaces(const Weight& w) {
  std::lock_guard<std::mutex> lock(g_ws_create_mu);
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
                         tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st,
                         float* ws, int* counters, int64_t ws_capacity_floats, int64_t ctr_capacity) {
  const GemvPlan pl = plan_gemv(w, m);
  GemvArgs args{};
  args.q = static_cast<const uint8_t*>(w.q.ptr);
  args.row_bytes = w.row_bytes;
  args.scales = w.scales.ptr;
  args.zps = w.zps.ptr;
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
  args.ctas_n = pl.ctas_n;
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
  const int tiles = pl.ctas_n * pl.ksplit;
  const int st_bytes = w.desc.dequant_dtype == TQ4_F32 ? 4 : 2;
  cudaError_t e;
  if (w.desc.bits == 4) e = launch_gemv_bits<4>(args, a_t, st_bytes, pl.mt, tiles, w.num_sms, pl.smem, st);
  else if (w.desc.bits == 2) e = launch_gemv_bits<2>(args, a_t, st_bytes, pl.mt, tiles, w.num_sms, pl.smem, st);
  else e = launch_gemv_bits<8>(args, a_t, st_bytes, pl.mt, tiles, w.num_sms, pl.smem, st);
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
