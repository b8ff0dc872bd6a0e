// Prefill-shaped MatMulNBits calls (M > 16): a warp-specialised tcgen05 GEMM that dequantizes the
// packed weight tiles in shared memory.
//
//   Y[M, N] = A[M, K] . W^T,  W = (q - z) * s  (dequantize_weight/4, quantized.ex:234-240)
//
// CTA tile 128 (M) x BN (N), one 64-byte packed group (128 4-bit weights) of K per stage, 2-4
// stages (as many as fit shared memory):
//   warp 0   TMA producer: A tile (two 64-column boxes, 128B swizzle), the packed W tile
//            (BN rows x 64 bytes) and the stage's block-major scales / zero points (BN rows x
//            the stage's blocks) into stage s, completing on full[s].
//   warp 1   TMEM allocation, and one thread that issues tcgen05.mma (M=128, N=BN, K=16) x 8
//            per stage into the f32 accumulator in TMEM; tcgen05.commit frees the stage.
//   warps 2-9 dequantize the packed tile into the MMA operand (A's type; W = RN_T(RN_T(q-z)*s)
//            exactly as the reference when T is A's type) in the 128B-swizzled K-major layout,
//            then run the epilogue: tcgen05.ld of their 32 TMEM lanes (warps w and w+4 split the
//            columns), bias, conversion, vector stores.
// Every mbarrier wait is bounded by a clock deadline; a wait that runs out writes the device
// status word, raises the CTA's abort flag and the CTA winds down (no trap, no endless spin).
#include "internal.cuh"
#include "sm100.cuh"

namespace tq4 {

// ---- PTX wrappers (mbarrier / TMA in sm100.cuh) ---------------------------------------------------
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  // K-major, 128-byte swizzle: LBO 16 B (unused inside one atom), SBO 1024 B (8 rows x 128 B),
  // version 1 (sm_100), layout type 2 (SWIZZLE_128B), base offset 0 (1024-aligned atoms).
  return (uint64_t)((addr & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)64 << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b, bool bf) {
  uint32_t r;
  if (bf) asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b, bool bf) {
  uint32_t r;
  if (bf) asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t h2_splat(float v, bool bf) {
  if (bf) {
    const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    return h | (h << 16);
  }
  const uint32_t h = __half_as_ushort(__float2half_rn(v));
  return h | (h << 16);
}

// q values of a 4-bit step (pair (e0,e1) -> p0, (e2,e3) -> p1) as exact small integers in the
// MMA type (f16 magic 1024 / bf16 magic 128, see common.cuh for the nibble order).
__device__ __forceinline__ void q_pairs4(uint32_t x, int j, bool bf, uint32_t& p0, uint32_t& p1) {
  const uint32_t src = (j & 1) ? (x >> 8) : x;
  if (!bf) {
    p0 = h2_sub(lop3_and_or(src, 0x000F000Fu, 0x64006400u), 0x64006400u, false);
    uint32_t r1 = lop3_and_or(src, 0x00F000F0u, 0x64006400u), out;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(r1), "r"(0x2C002C00u), "r"(0xD400D400u));
    p1 = out;
  } else {
    p0 = h2_sub(lop3_and_or(src, 0x000F000Fu, 0x43004300u), 0x43004300u, true);
    p1 = h2_sub(lop3_and_or(src >> 4, 0x000F000Fu, 0x43004300u), 0x43004300u, true);
  }
}

// (q - z) * s of one pair in the MMA type. T_SAME: T is the MMA type (exact reference math in
// packed f16x2/bf16x2); otherwise computed in f32 with T's roundings, then converted.
template <bool BF, tq4_dtype T>
__device__ __forceinline__ uint32_t deq_pair(uint32_t qp, float z, float s) {
  constexpr bool T_SAME = (BF && T == TQ4_BF16) || (!BF && T == TQ4_F16);
  if constexpr (T_SAME) {
    return h2_mul(h2_sub(qp, h2_splat(z, BF), BF), h2_splat(s, BF), BF);
  } else {
    float q0, q1;
    if (BF) {
      q0 = __uint_as_float(qp << 16);
      q1 = __uint_as_float(qp & 0xFFFF0000u);
    } else {
      q0 = __half2float(__ushort_as_half((uint16_t)(qp & 0xFFFF)));
      q1 = __half2float(__ushort_as_half((uint16_t)(qp >> 16)));
    }
    float w0, w1;
    if constexpr (T == TQ4_F32) {
      w0 = __fmul_rn(__fsub_rn(q0, z), s);
      w1 = __fmul_rn(__fsub_rn(q1, z), s);
    } else {
      w0 = round_to(round_to((float)((double)q0 - (double)z), T) * s, T);
      w1 = round_to(round_to((float)((double)q1 - (double)z), T) * s, T);
    }
    if (BF) {
      __nv_bfloat162 h = __floats2bfloat162_rn(w0, w1);
      return *reinterpret_cast<uint32_t*>(&h);
    }
    __half2 h = __floats2half2_rn(w0, w1);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}


struct GemmArgs {
  float z_const;
  int has_zp;
  int bs_log2;
  int nb;          // scale blocks per stage (the TMA box height)
  int M, N, K;
  int ktiles;      // 64-byte groups per row
  int stages;
  int stage_bytes;
  int sc_off, zc_off;  // offsets of the staged scales / zero points within a stage
  int st_bytes;
  int int_zp;      // zero points are integers (packed or absent): the fused dequant path applies
  const void* bias;
  tq4_dtype bias_t;
  void* y;
  tq4_dtype y_t;
  int64_t ldy;
};

constexpr int kGemmThreads = 320;  // producer, MMA, 8 dequant / epilogue warps
constexpr int BM = 128;
constexpr int kMaxStages = 4;

template <int BN>
struct GemmTile {
  static constexpr int A_BYTES = BM * 128 * 2;    // 128 rows x 128 k x 2 B (two SW128 halves)
  static constexpr int W16_BYTES = BN * 128 * 2;  // BN rows x 128 k x 2 B (two SW128 halves)
  static constexpr int WP_BYTES = BN * 64;        // packed
  static constexpr int FIXED = A_BYTES + W16_BYTES + WP_BYTES;
  static constexpr int TMEM_COLS = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
};

template <int BN, bool BF, tq4_dtype T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_z,
                const GemmArgs p) {
  using L = GemmTile<BN>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const int S = p.stages;
  const uint32_t bars = base + S * p.stage_bytes;
  auto full = [&](int s) { return bars + 8 * s; };
  auto deq = [&](int s) { return bars + 8 * (kMaxStages + s); };
  auto empty = [&](int s) { return bars + 8 * (2 * kMaxStages + s); };
  const uint32_t accum = bars + 8 * (3 * kMaxStages);
  uint8_t* tail = smem + S * p.stage_bytes + 8 * (3 * kMaxStages + 1);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(tail);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tail + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int KT = p.ktiles;
  const uint32_t tx_bytes = L::A_BYTES + L::WP_BYTES + BN * p.nb * p.st_bytes * (p.has_zp ? 2 : 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(deq(s), 256);
      mbar_init(empty(s), 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)tmem_slot)), "r"((uint32_t)L::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % S;
        const uint32_t ph = (kt / S) & 1;
        if (!mbar_wait(empty(s), ph ^ 1, abort_flag, kDevTimeoutStageEmpty)) break;
        const uint32_t st = base + s * p.stage_bytes;
        const int b0 = (kt * 128) >> p.bs_log2;
        mbar_expect_tx(full(s), tx_bytes);
        tma_load_2d(st, &map_a, kt * 128, m0, full(s));
        tma_load_2d(st + L::A_BYTES / 2, &map_a, kt * 128 + 64, m0, full(s));
        tma_load_2d(st + L::A_BYTES + L::W16_BYTES, &map_w, kt * 64, n0, full(s));
        tma_load_2d(st + p.sc_off, &map_s, n0, b0, full(s));
        if (p.has_zp) tma_load_2d(st + p.zc_off, &map_z, n0, b0, full(s));
        issued = kt + 1;
      }
      // the copies still in flight complete before the CTA exits (bounded)
      for (int kt = max(0, issued - S); kt < issued; ++kt) {
        const long long t0 = clock64();
        while (!mbar_try(full(kt % S), (kt / S) & 1) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | ((BF ? 1u : 0u) << 7) | ((BF ? 1u : 0u) << 10) |
                                 ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      bool ok = true;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int s = kt % S;
        const uint32_t ph = (kt / S) & 1;
        ok = mbar_wait(full(s), ph, abort_flag, kDevTimeoutTmaFull) &&
             mbar_wait(deq(s), ph, abort_flag, kDevTimeoutDequant);
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t a_base = base + s * p.stage_bytes;
        const uint32_t w_base = a_base + L::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t h = kk >> 2, off = (kk & 3) * 32;
          const uint64_t ad = smem_desc_sw128(a_base + h * (L::A_BYTES / 2) + off);
          const uint64_t bd = smem_desc_sw128(w_base + h * (L::W16_BYTES / 2) + off);
          mma_f16(tmem, ad, bd, idesc, (kt | kk) != 0);
        }
        mma_commit(empty(s));
      }
      mma_commit(accum);  // also after an abort: the epilogue waits for the issued MMAs
    }
  } else {
    // ---------------- dequant warps (then epilogue) ----------------
    const int tid = threadIdx.x - 64;  // 0..255
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % S;
      const uint32_t ph = (kt / S) & 1;
      if (!mbar_wait(full(s), ph, abort_flag, kDevTimeoutTmaFull)) break;
      uint8_t* st = smem + s * p.stage_bytes;
      const uint8_t* wp = st + L::A_BYTES + L::W16_BYTES;
      uint8_t* w16 = st + L::A_BYTES;
      const uint8_t* sc = st + p.sc_off;
      const uint8_t* zc = st + p.zc_off;
      const int b0 = (kt * 128) >> p.bs_log2;
      constexpr bool T_SAME = (BF && T == TQ4_BF16) || (!BF && T == TQ4_F16);
      for (int task = tid; task < BN * 4; task += 256) {
        const int r = task >> 2, t = task & 3;
        const uint4 v = *reinterpret_cast<const uint4*>(wp + r * 64 + t * 16);
        if constexpr (T_SAME) {
          if (p.int_zp) {
            // T is the MMA type and the zero points are integers: (O + q) - (O + z) is exact, so
            // one f16x2/bf16x2 op gives q - z straight from the magic-number value, and one more
            // multiply gives RN_T((q - z) * s), the reference's weight.
            const uint16_t* sc16 = reinterpret_cast<const uint16_t*>(sc);
            const uint16_t* zc16 = reinterpret_cast<const uint16_t*>(zc);
            uint32_t s2 = 0, oz2 = 0, oz16 = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (j == 0 || ((16 * j) & ((1 << p.bs_log2) - 1)) == 0) {  // a new block
                const int lb = ((kt * 128 + 16 * j) >> p.bs_log2) - b0;
                const uint32_t sv = sc16[lb * BN + r];
                s2 = sv | (sv << 16);
                const float z = p.has_zp ? scale_to_f32(zc16, lb * BN + r, 2, BF) : p.z_const;
                oz2 = h2_splat((BF ? 128.f : 1024.f) + z, BF);  // O + z (exact)
                oz16 = h2_splat(64.f + z, BF);                   // for the 16q pair (f16)
              }
              const uint32_t x = (j < 2) ? v.x : (j < 4) ? v.y : (j < 6) ? v.z : v.w;
              const uint32_t src = (j & 1) ? (x >> 8) : x;
              uint32_t d0, d1;
              if (!BF) {
                d0 = h2_sub(lop3_and_or(src, 0x000F000Fu, 0x64006400u), oz2, false);
                const uint32_t r1 = lop3_and_or(src, 0x00F000F0u, 0x64006400u);  // 1024 + 16 q
                // r1/16 - (64 + z) = q - z, one rounding of an exact value
                asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d1) : "r"(r1), "r"(0x2C002C00u), "r"(oz16 ^ 0x80008000u));
              } else {
                d0 = h2_sub(lop3_and_or(src, 0x000F000Fu, 0x43004300u), oz2, true);
                d1 = h2_sub(lop3_and_or(src >> 4, 0x000F000Fu, 0x43004300u), oz2, true);
              }
              uint2 out;
              out.x = h2_mul(d0, s2, BF);
              out.y = h2_mul(d1, s2, BF);
              const int chunk = 2 * (j & 3) + (t >> 1);
              uint8_t* dst = w16 + (j >> 2) * (BN * 128) + r * 128 + ((chunk ^ (r & 7)) << 4) + ((t & 1) << 3);
              *reinterpret_cast<uint2*>(dst) = out;
            }
            continue;
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t x = (j < 2) ? v.x : (j < 4) ? v.y : (j < 6) ? v.z : v.w;
          const int lb = ((kt * 128 + 16 * j) >> p.bs_log2) - b0;  // staged block row
          const float scv = scale_to_f32(sc, lb * BN + r, p.st_bytes, T == TQ4_BF16);
          const float z = p.has_zp ? scale_to_f32(zc, lb * BN + r, p.st_bytes, T == TQ4_BF16) : p.z_const;
          uint32_t q0, q1;
          q_pairs4(x, j, BF, q0, q1);
          uint2 out;
          out.x = deq_pair<BF, T>(q0, z, scv);
          out.y = deq_pair<BF, T>(q1, z, scv);
          // k within the group = 16j + 4t: half j/4, 16-byte chunk 2(j%4) + t/2, 8-byte half t%2
          const int chunk = 2 * (j & 3) + (t >> 1);
          uint8_t* dst = w16 + (j >> 2) * (BN * 128) + r * 128 + ((chunk ^ (r & 7)) << 4) + ((t & 1) << 3);
          *reinterpret_cast<uint2*>(dst) = out;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(deq(s));
    }

    // ---------------- epilogue ----------------
    const long long t0 = clock64();
    bool ok = true;
    while (!mbar_try(accum, 0)) {
      if (clock64() - t0 > kWaitCycles) {
        report(kDevTimeoutAccum);
        *abort_flag = 1;
        ok = false;
        break;
      }
    }
    asm volatile("tcgen05.fence::after_thread_sync;");
    const int quarter = warp & 3;                // TMEM lanes 32*quarter .. +31
    const int half = (warp - 2) >> 2;            // columns [half*BN/2, (half+1)*BN/2)
    const int row = m0 + quarter * 32 + lane;
    if (__all_sync(0xffffffffu, ok && !*abort_flag)) {
#pragma unroll 1
      for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + c, r);
        if (row < p.M) {
          const int64_t nb0 = (int64_t)n0 + c;
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            v[i] = __uint_as_float(r[i]);
            if (p.bias && nb0 + i < p.N) v[i] = round_to(v[i], p.y_t) + load_as_f32(p.bias, nb0 + i, p.bias_t);
          }
          const int64_t off = (int64_t)row * p.ldy + nb0;
          const bool whole = nb0 + 16 <= p.N;
          const uintptr_t addr = reinterpret_cast<uintptr_t>(p.y) + off * (p.y_t == TQ4_F32 ? 4 : 2);
          const bool aligned = (addr & 15) == 0;  // 16-byte vector stores
          if (whole && aligned && p.y_t != TQ4_F32) {
            uint32_t h[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              if (p.y_t == TQ4_BF16) {
                __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                h[i] = *reinterpret_cast<uint32_t*>(&b2);
              } else {
                __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
                h[i] = *reinterpret_cast<uint32_t*>(&h2);
              }
            }
            uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.y) + off);
            dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
            dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
          } else if (whole && aligned && p.y_t == TQ4_F32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.y) + off);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (nb0 + i < p.N) store_from_f32(p.y, off + i, p.y_t, v[i]);
          }
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
  }

  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)L::TMEM_COLS));
  }
}

// ---- host side ---------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

tq4_status make_map(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t inner,
                    uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return TQ4_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TQ4_ERR_CUDA;
  }
  return TQ4_OK;
}

static const int kTileWidths[3] = {128, 96, 64};

static int gemm_scale_blocks(const Weight& w) { return std::max(1, 128 >> w.bs_log2); }

// Descriptors of a new handle, one set per GEMM tile width (4-bit weights only): the packed rows
// (box BN x 64 bytes) and the block-major scales / zero points (box BN rows x the stage's blocks).
tq4_status make_weight_maps(Weight& w) {
  w.wmaps_ok = false;
  if (w.desc.bits != 4 || encode_fn() == nullptr) return TQ4_OK;
  const int st = dtype_size(w.desc.dequant_dtype);
  const CUtensorMapDataType sdt = st == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const int nb = gemm_scale_blocks(w);
  for (int i = 0; i < 3; ++i) {
    const int bn = kTileWidths[i];
    TQ4_TRY(make_map(&w.wmaps[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q.ptr, w.row_bytes, w.n_pad,
                     w.row_bytes, 64, bn, CU_TENSOR_MAP_SWIZZLE_NONE));
    TQ4_TRY(make_map(&w.smaps[i], sdt, w.scales.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, bn, nb,
                     CU_TENSOR_MAP_SWIZZLE_NONE));
    if (w.zps.ptr)
      TQ4_TRY(make_map(&w.zmaps[i], sdt, w.zps.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, bn, nb,
                       CU_TENSOR_MAP_SWIZZLE_NONE));
    else
      w.zmaps[i] = w.smaps[i];  // never loaded
  }
  w.wmaps_ok = true;
  return TQ4_OK;
}

constexpr int kSmemLimit = 232448;  // 227 KB of dynamic shared memory per CTA

struct GemmPlan {
  int stages, stage_bytes, sc_off, zc_off, smem;
};

template <int BN>
static GemmPlan plan_gemm_smem(const Weight& w) {
  using L = GemmTile<BN>;
  GemmPlan pl{};
  const int st = dtype_size(w.desc.dequant_dtype);
  const int sc_bytes = BN * gemm_scale_blocks(w) * st;
  pl.sc_off = L::FIXED;
  pl.zc_off = pl.sc_off + (sc_bytes + 127) / 128 * 128;
  const int end = pl.zc_off + (w.zps.ptr ? sc_bytes : 0);
  pl.stage_bytes = (end + 1023) / 1024 * 1024;
  const int fixed = 1024 + 8 * (3 * kMaxStages + 1) + 16;
  pl.stages = std::min(kMaxStages, (kSmemLimit - fixed) / pl.stage_bytes);
  pl.smem = fixed + pl.stages * pl.stage_bytes;
  return pl;
}

template <int BN, bool BF, tq4_dtype T>
static tq4_status launch_gemm_t(const CUtensorMap& ma, const Weight& w, int map_i, GemmArgs args,
                                cudaStream_t st) {
  const GemmPlan pl = plan_gemm_smem<BN>(w);
  if (pl.stages < 2) {
    set_error("GEMM: the stage does not fit shared memory");
    return TQ4_ERR_UNSUPPORTED;
  }
  args.stages = pl.stages;
  args.stage_bytes = pl.stage_bytes;
  args.sc_off = pl.sc_off;
  args.zc_off = pl.zc_off;
  auto kern = gemm_kernel<BN, BF, T>;
  static bool attr_set = false;  // once per instantiation, at the largest size it can ask for
  if (!attr_set) {
    TQ4_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    attr_set = true;
  }
  const dim3 grid((args.N + BN - 1) / BN, (args.M + BM - 1) / BM);
  kern<<<grid, kGemmThreads, pl.smem, st>>>(ma, w.wmaps[map_i], w.smaps[map_i], w.zmaps[map_i], args);
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

template <int BN, bool BF>
static tq4_status launch_gemm_bn(const CUtensorMap& ma, const Weight& w, int map_i,
                                 const GemmArgs& args, cudaStream_t st) {
  switch (w.desc.dequant_dtype) {
    case TQ4_F16: return launch_gemm_t<BN, BF, TQ4_F16>(ma, w, map_i, args, st);
    case TQ4_BF16: return launch_gemm_t<BN, BF, TQ4_BF16>(ma, w, map_i, args, st);
    default: return launch_gemm_t<BN, BF, TQ4_F32>(ma, w, map_i, args, st);
  }
}

// Whether the tcgen05 GEMM takes this call (else A goes through the GEMV in 16-row slices).
static bool gemm_eligible(const Weight& w, const void* a, tq4_dtype a_t) {
  if (w.desc.bits != 4) return false;
  if (a_t != TQ4_F16 && a_t != TQ4_BF16) return false;
  if ((w.desc.K * 2) % 16 != 0) return false;                    // TMA row stride
  if ((reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;  // TMA base address
  return w.wmaps_ok;
}

static int choose_bn(const Weight& w, int64_t m) {
  // fill the SMs: prefer the widest tile whose grid still covers them
  const int64_t mt = (m + BM - 1) / BM;
  const int sms = w.num_sms;
  for (int bn : kTileWidths) {
    const int64_t tiles = mt * ((w.desc.N + bn - 1) / bn);
    if (tiles >= sms * 3 / 4) return bn;
  }
  return 64;
}

tq4_status run_gemm_tc(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                       tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  const int bn = choose_bn(w, m);
  const int map_i = bn == 128 ? 0 : (bn == 96 ? 1 : 2);
  CUtensorMap ma;
  const CUtensorMapDataType adt = a_t == TQ4_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  TQ4_TRY(make_map(&ma, adt, a, w.desc.K, m, w.desc.K * 2, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B));
  GemmArgs args{};
  args.z_const = w.z_const;
  args.has_zp = w.zps.ptr != nullptr;
  args.bs_log2 = w.bs_log2;
  args.nb = gemm_scale_blocks(w);
  args.M = (int)m;
  args.N = (int)w.desc.N;
  args.K = (int)w.desc.K;
  args.ktiles = (int)w.groups;
  args.st_bytes = dtype_size(w.desc.dequant_dtype);
  args.int_zp = w.desc.zp_kind != TQ4_ZP_FLOAT;
  args.bias = bias;
  args.bias_t = bias_t;
  args.y = y;
  args.y_t = y_t;
  args.ldy = ldy;
  const bool bf = a_t == TQ4_BF16;
  if (bn == 128) return bf ? launch_gemm_bn<128, true>(ma, w, map_i, args, st) : launch_gemm_bn<128, false>(ma, w, map_i, args, st);
  if (bn == 96) return bf ? launch_gemm_bn<96, true>(ma, w, map_i, args, st) : launch_gemm_bn<96, false>(ma, w, map_i, args, st);
  return bf ? launch_gemm_bn<64, true>(ma, w, map_i, args, st) : launch_gemm_bn<64, false>(ma, w, map_i, args, st);
}

// Rows of A in slices of 16 through the fused GEMV kernel (2- and 8-bit weights, f32
// activations, and A that TMA cannot address).
static tq4_status run_gemm_by_slices(const Weight& w, const void* a, int64_t m, tq4_dtype a_t,
                                     const void* bias, tq4_dtype bias_t, void* y, tq4_dtype y_t,
                                     int64_t ldy, cudaStream_t st) {
  const int as = dtype_size(a_t), ys = dtype_size(y_t);
  for (int64_t r = 0; r < m; r += 16) {
    const int64_t rows = std::min<int64_t>(16, m - r);
    TQ4_TRY(run_gemv(w, static_cast<const uint8_t*>(a) + r * w.desc.K * as, rows, a_t, bias,
                     bias_t, static_cast<uint8_t*>(y) + r * ldy * ys, y_t, ldy, st));
  }
  return TQ4_OK;
}

tq4_status run_gemm(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                    tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  if (gemm_eligible(w, a, a_t)) return run_gemm_tc(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
  return run_gemm_by_slices(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
}

tq4_status run_matmul(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                      tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  if (m <= 16) return run_gemv(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
  return run_gemm(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
}

}  // namespace tq4
