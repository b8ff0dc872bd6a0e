// MMA fragment helpers shared by the GEMV kernels (gemv.cu, gemv_rows.cu): the magic-number
// weight pairs of the packed layout (common.cuh), the activation factors that match them, the
// legacy-path mma.sync m16n8k16 wrapper and the activation loads.
#pragma once

#include "common.cuh"

namespace tq4 {

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
// weight at position k (k counted from the start of a 64-byte group).
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

// 1 / act_factor (a power of two).
template <int BITS, bool BF, bool PRECISE>
__device__ __forceinline__ float act_factor_inv(int k) {
  if constexpr (BF) return 1.f;
  if constexpr (BITS == 4 && PRECISE) return 16.f;
  if constexpr (BITS == 4) return (k & 2) ? 16.f : 1.f;
  if constexpr (BITS == 2 && PRECISE) return 1.f;
  if constexpr (BITS == 2) {
    const int i = 2 * ((k >> 4) & 1) + ((k >> 1) & 1);
    return i == 0 ? 1.f : (i == 1 ? 4.f : (i == 2 ? 16.f : 64.f));
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

__device__ __forceinline__ uint32_t word_of(const uint4& v, int w) {
  return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
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

}  // namespace tq4
