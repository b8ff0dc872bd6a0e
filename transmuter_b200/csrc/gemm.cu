// Prefill-shaped MatMulNBits calls (M > 16): a warp-specialised tcgen05 GEMM whose dequantised
// weights are the MMA's A operand in tensor memory.
//
//   Y[M, N] = A[M, K] . W^T,  W = (q - z) * s  (dequantize_weight/4, quantized.ex:234-240)
//
// computed as Y^T tile = W tile . A tile^T: a CTA takes 128 weight rows (the MMA's M, one TMEM
// lane each) and TM activation rows (the MMA's N, 32..256). Per stage of 128 k (one 64-byte
// packed group):
//   warp 0   TMA producer: the activation tile (two 64-k boxes, 128B swizzle: the K-major B
//            operand), the packed weight tile (128 rows x 64 bytes) and the stage's block-major
//            scales / zero points, completing on full[s].
//   warps 2-9 dequantise in registers: warp w owns TMEM lanes 32*(w%4).. (its 32 weight rows)
//            and one half of the stage's k; each thread turns its row's 64 weights into
//            RN_T(RN_T(q - z) * s) (exactly the reference's weight when T is A's type) and
//            writes them with tcgen05.st into one of 4 TMEM weight slots (64 columns each).
//   warp 1   TMEM allocation, and one thread that issues tcgen05.mma (M=128, N=TM, K=16, A from
//            TMEM, B from shared memory) x 8 per stage into the f32 accumulator (TM columns);
//            tcgen05.commit frees the shared-memory stage and the TMEM slot.
//   warps 2-9 then run the epilogue: tcgen05.ld of their lanes (one weight row, consecutive
//            activation rows), bias, conversion, stores (a warp writes 32 consecutive columns).
// The shared-memory ring (2-4 stages) and the TMEM slot ring (4) are independent, so the copies,
// the dequantisation and the MMAs overlap instead of paying their latencies in sequence.
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



// tcgen05.mma with the A operand in tensor memory.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
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
constexpr int WN = 128;            // weight rows per CTA: the MMA's M and the TMEM lanes
constexpr int kMaxStages = 4;      // shared-memory stages
constexpr int kASlots = 4;         // dequantised weight stages in TMEM, 64 columns each
constexpr int kTmemCols = 512;

template <int TM>
struct GemmTile {
  static constexpr int ACT_BYTES = TM * 128 * 2;  // TM rows x 128 k x 2 B (two SW128 halves)
  static constexpr int WP_BYTES = WN * 64;        // packed
  static constexpr int FIXED = ACT_BYTES + WP_BYTES;
  static_assert(TM % 32 == 0 && TM >= 32 && TM <= 256, "MMA N");
  static_assert(TM + kASlots * 64 <= kTmemCols, "TMEM columns");
};

template <int TM, bool BF, tq4_dtype T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_z,
                const GemmArgs p) {
  using L = GemmTile<TM>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const int S = p.stages;
  const uint32_t bars = base + S * p.stage_bytes;
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (kMaxStages + s); };
  auto afull = [&](int a) { return bars + 8 * (2 * kMaxStages + a); };
  auto aempty = [&](int a) { return bars + 8 * (2 * kMaxStages + kASlots + a); };
  const uint32_t accum = bars + 8 * (2 * kMaxStages + 2 * kASlots);
  uint8_t* tail = smem + S * p.stage_bytes + 8 * (2 * kMaxStages + 2 * kASlots + 1);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(tail);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tail + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * WN, m0 = blockIdx.y * TM;
  const int KT = p.ktiles;
  const uint32_t tx_bytes = L::FIXED + WN * p.nb * p.st_bytes * (p.has_zp ? 2 : 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1 + 8);  // the MMAs' commit + the 8 dequantising warps
    }
    for (int a = 0; a < kASlots; ++a) {
      mbar_init(afull(a), 8);
      mbar_init(aempty(a), 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)tmem_slot)), "r"((uint32_t)kTmemCols));
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
        tma_load_2d(st + L::ACT_BYTES / 2, &map_a, kt * 128 + 64, m0, full(s));
        tma_load_2d(st + L::ACT_BYTES, &map_w, kt * 64, n0, full(s));
        tma_load_2d(st + p.sc_off, &map_s, n0, b0, full(s));
        if (p.has_zp) tma_load_2d(st + p.zc_off, &map_z, n0, b0, full(s));
        issued = kt + 1;
      }
      // the copies still in flight complete before the CTA exits (bounded)
      for (int kt = max(0, issued - S); kt < issued; ++kt) mbar_drain(full(kt % S), (kt / S) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | ((BF ? 1u : 0u) << 7) | ((BF ? 1u : 0u) << 10) |
                                 ((uint32_t)(TM >> 3) << 17) | ((uint32_t)(WN >> 4) << 24);
      bool ok = true;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int s = kt % S, a = kt % kASlots;
        ok = mbar_wait(full(s), (kt / S) & 1, abort_flag, kDevTimeoutTmaFull) &&
             mbar_wait(afull(a), (kt / kASlots) & 1, abort_flag, kDevTimeoutDequant);
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t act = base + s * p.stage_bytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t h = kk >> 2, off = (kk & 3) * 32;
          const uint64_t bd = smem_desc_sw128(act + h * (L::ACT_BYTES / 2) + off);
          mma_ts(tmem, tmem + TM + a * 64 + kk * 8, bd, idesc, (kt | kk) != 0);
        }
        mma_commit(empty(s));
        mma_commit(aempty(a));
      }
      mma_commit(accum);  // also after an abort: the epilogue waits for the issued MMAs
    }
  } else {
    // ---------------- dequantising warps (then epilogue) ----------------
    const int quarter = warp & 3;          // TMEM lanes 32*quarter .. +31
    const int khalf = (warp - 2) >> 2;     // k 64*khalf .. +63 of each stage
    const int r = quarter * 32 + lane;     // this thread's weight row in the tile
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    constexpr bool T_SAME = (BF && T == TQ4_BF16) || (!BF && T == TQ4_F16);
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % S, a = kt % kASlots;
      if (!mbar_wait(full(s), (kt / S) & 1, abort_flag, kDevTimeoutTmaFull)) break;
      if (!mbar_wait(aempty(a), ((kt / kASlots) & 1) ^ 1, abort_flag, kDevTimeoutDequant)) break;
      const uint8_t* st = smem + s * p.stage_bytes;
      const uint8_t* wp = st + L::ACT_BYTES + r * 64 + khalf * 8;
      const uint8_t* sc = st + p.sc_off;
      const uint8_t* zc = st + p.zc_off;
      // words 2*khalf and 2*khalf+1 of the row's four 16-byte pieces: steps 4*khalf .. +3
      uint2 v[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) v[t] = *reinterpret_cast<const uint2*>(wp + t * 16);
      const int b0 = (kt * 128) >> p.bs_log2;
      uint32_t out[32];  // column c holds k = 64*khalf + 2c, 2c + 1
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = 4 * khalf + jj;
        const int lb = ((kt * 128 + 16 * j) >> p.bs_log2) - b0;  // staged block row
        if (T_SAME && p.int_zp) {
          // (O + q) - (O + z) is exact in the MMA type; one more multiply gives RN_T((q - z) * s)
          const uint16_t* sc16 = reinterpret_cast<const uint16_t*>(sc);
          const uint32_t sv = sc16[lb * WN + r];
          const uint32_t s2 = sv | (sv << 16);
          const float z = p.has_zp ? scale_to_f32(zc, lb * WN + r, 2, BF) : p.z_const;
          const uint32_t oz2 = h2_splat((BF ? 128.f : 1024.f) + z, BF);
          const uint32_t oz16n = h2_splat(-(64.f + z), BF);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t x = (jj < 2) ? v[t].x : v[t].y;
            const uint32_t src = (jj & 1) ? (x >> 8) : x;
            uint32_t d0, d1;
            if (!BF) {
              d0 = h2_sub(lop3_and_or(src, 0x000F000Fu, 0x64006400u), oz2, false);
              const uint32_t r1 = lop3_and_or(src, 0x00F000F0u, 0x64006400u);  // 1024 + 16 q
              asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d1) : "r"(r1), "r"(0x2C002C00u), "r"(oz16n));
            } else {
              d0 = h2_sub(lop3_and_or(src, 0x000F000Fu, 0x43004300u), oz2, true);
              d1 = h2_sub(lop3_and_or(src >> 4, 0x000F000Fu, 0x43004300u), oz2, true);
            }
            out[8 * jj + 2 * t] = h2_mul(d0, s2, BF);
            out[8 * jj + 2 * t + 1] = h2_mul(d1, s2, BF);
          }
        } else {
          const float scv = scale_to_f32(sc, lb * WN + r, p.st_bytes, T == TQ4_BF16);
          const float z = p.has_zp ? scale_to_f32(zc, lb * WN + r, p.st_bytes, T == TQ4_BF16) : p.z_const;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t x = (jj < 2) ? v[t].x : v[t].y;
            uint32_t q0, q1;
            q_pairs4(x, jj, BF, q0, q1);
            out[8 * jj + 2 * t] = deq_pair<BF, T>(q0, z, scv);
            out[8 * jj + 2 * t + 1] = deq_pair<BF, T>(q1, z, scv);
          }
        }
      }
      tmem_st32(lane_addr + TM + a * 64 + khalf * 32, out);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(afull(a));
        mbar_arrive(empty(s));
      }
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
    const int chalf = khalf;  // activation rows [chalf*TM/2, (chalf+1)*TM/2) of the tile
    const int64_t n = (int64_t)n0 + r;
    const bool n_ok = n < p.N;
    const float bias_v = (p.bias && n_ok) ? load_as_f32(p.bias, n, p.bias_t) : 0.f;
    if (__all_sync(0xffffffffu, ok && !*abort_flag)) {
#pragma unroll 1
      for (int c = chalf * (TM / 2); c < (chalf + 1) * (TM / 2); c += 16) {
        uint32_t rr[16];
        tmem_ld16(lane_addr + c, rr);
        if (n_ok) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int64_t m = (int64_t)m0 + c + i;
            if (m < p.M) {
              float v = __uint_as_float(rr[i]);
              if (p.bias) v = round_to(v, p.y_t) + bias_v;
              store_from_f32(p.y, m * p.ldy + n, p.y_t, v);
            }
          }
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
  }

  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTmemCols));
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

static int gemm_scale_blocks(const Weight& w) { return std::max(1, 128 >> w.bs_log2); }

// Descriptors of a new handle (4-bit weights only): the packed rows (box 128 rows x 64 bytes) and
// the block-major scales / zero points (box 128 rows x the stage's blocks).
tq4_status make_weight_maps(Weight& w) {
  w.wmaps_ok = false;
  if (w.desc.bits != 4 || encode_fn() == nullptr) return TQ4_OK;
  const int st = dtype_size(w.desc.dequant_dtype);
  const CUtensorMapDataType sdt = st == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const int nb = gemm_scale_blocks(w);
  TQ4_TRY(make_map(&w.wmaps[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q.ptr, w.row_bytes, w.n_pad, w.row_bytes, 64,
                   WN, CU_TENSOR_MAP_SWIZZLE_NONE));
  TQ4_TRY(make_map(&w.smaps[0], sdt, w.scales.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, WN, nb,
                   CU_TENSOR_MAP_SWIZZLE_NONE));
  if (w.zps.ptr)
    TQ4_TRY(make_map(&w.zmaps[0], sdt, w.zps.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, WN, nb,
                     CU_TENSOR_MAP_SWIZZLE_NONE));
  else
    w.zmaps[0] = w.smaps[0];  // never loaded
  w.wmaps_ok = true;
  return TQ4_OK;
}

constexpr int kSmemLimit = 232448;  // 227 KB of dynamic shared memory per CTA

struct GemmPlan {
  int stages, stage_bytes, sc_off, zc_off, smem;
};

template <int TM>
static GemmPlan plan_gemm_smem(const Weight& w) {
  using L = GemmTile<TM>;
  GemmPlan pl{};
  const int st = dtype_size(w.desc.dequant_dtype);
  const int sc_bytes = WN * gemm_scale_blocks(w) * st;
  pl.sc_off = L::FIXED;
  pl.zc_off = pl.sc_off + (sc_bytes + 127) / 128 * 128;
  const int end = pl.zc_off + (w.zps.ptr ? sc_bytes : 0);
  pl.stage_bytes = (end + 1023) / 1024 * 1024;
  const int fixed = 1024 + 8 * (2 * kMaxStages + 2 * kASlots + 1) + 16;
  pl.stages = std::min(kMaxStages, (kSmemLimit - fixed) / pl.stage_bytes);
  pl.smem = fixed + pl.stages * pl.stage_bytes;
  return pl;
}

template <int TM, bool BF, tq4_dtype T>
static tq4_status launch_gemm_t(const CUtensorMap& ma, const Weight& w, GemmArgs args, cudaStream_t st) {
  const GemmPlan pl = plan_gemm_smem<TM>(w);
  if (pl.stages < 2) {
    set_error("GEMM: the stage does not fit shared memory");
    return TQ4_ERR_UNSUPPORTED;
  }
  args.stages = pl.stages;
  args.stage_bytes = pl.stage_bytes;
  args.sc_off = pl.sc_off;
  args.zc_off = pl.zc_off;
  auto kern = gemm_kernel<TM, BF, T>;
  static bool attr_set = false;  // once per instantiation, at the largest size it can ask for
  if (!attr_set) {
    TQ4_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    attr_set = true;
  }
  const dim3 grid((args.N + WN - 1) / WN, (args.M + TM - 1) / TM);
  kern<<<grid, kGemmThreads, pl.smem, st>>>(ma, w.wmaps[0], w.smaps[0], w.zmaps[0], args);
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

template <int TM, bool BF>
static tq4_status launch_gemm_tm(const CUtensorMap& ma, const Weight& w, const GemmArgs& args, cudaStream_t st) {
  switch (w.desc.dequant_dtype) {
    case TQ4_F16: return launch_gemm_t<TM, BF, TQ4_F16>(ma, w, args, st);
    case TQ4_BF16: return launch_gemm_t<TM, BF, TQ4_BF16>(ma, w, args, st);
    default: return launch_gemm_t<TM, BF, TQ4_F32>(ma, w, args, st);
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

// Activation rows per CTA: the largest tile that still gives half the SMs a tile.
static int choose_tm(const Weight& w, int64_t m) {
  const int64_t nt = (w.desc.N + WN - 1) / WN;
  for (int tm : {256, 128, 64}) {
    if (((m + tm - 1) / tm) * nt >= w.num_sms / 2) return tm;
  }
  return 32;
}

tq4_status run_gemm_tc(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                       tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  const int tm = choose_tm(w, m);
  CUtensorMap ma;
  const CUtensorMapDataType adt = a_t == TQ4_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  TQ4_TRY(make_map(&ma, adt, a, w.desc.K, m, w.desc.K * 2, 64, tm, CU_TENSOR_MAP_SWIZZLE_128B));
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
  switch (tm) {
    case 256: return bf ? launch_gemm_tm<256, true>(ma, w, args, st) : launch_gemm_tm<256, false>(ma, w, args, st);
    case 128: return bf ? launch_gemm_tm<128, true>(ma, w, args, st) : launch_gemm_tm<128, false>(ma, w, args, st);
    case 64: return bf ? launch_gemm_tm<64, true>(ma, w, args, st) : launch_gemm_tm<64, false>(ma, w, args, st);
    default: return bf ? launch_gemm_tm<32, true>(ma, w, args, st) : launch_gemm_tm<32, false>(ma, w, args, st);
  }
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
