// Prefill-shaped MatMulNBits calls (M > 16): a warp-specialised tcgen05 GEMM whose dequantised
// weights are the MMA's A operand in tensor memory.
//
//   Y[M, N] = A[M, K] . W^T,  W = (q - z) * s  (dequantize_weight/4, quantized.ex:234-240)
//
// computed as Y^T tile = W tile . A tile^T: a CTA takes 128 weight rows (the MMA's M, one TMEM
// lane each) and TM activation rows (the MMA's N, 32..256). Per stage of 128 k (one 64-byte
// packed group of 4-bit weights; two groups of 8-bit weights; half a group of 2-bit weights,
// whose group of 256 k is loaded whole by both of its stages):
//   warp 0   TMA producer: the activation tile (two 64-k boxes, 128B swizzle: the K-major B
//            operand), the packed weight tile (128 rows x 64 bytes per group) and the stage's
//            block-major scales / zero points, completing on full[s].
//   warps 2-17 dequantise in registers: warp w owns TMEM lanes 32*(w%4).. (its 32 weight rows)
//            and 16-byte pieces of each row (32 weights each, spread over the stage's k; the
//            packed tile arrives with the 64-byte swizzle, so these loads are free of bank
//            conflicts): with 256-row activation tiles all 16 warps take every stage, one piece
//            each; with narrower tiles two teams of 8 take alternate stages, two pieces each.
//            Each thread turns them into RN_T(RN_T(q - z) * s) (exactly the reference's weight
//            when T is A's type) and writes them with tcgen05.st into one of 4 TMEM weight slots
//            (64 columns each).
//   warp 1   TMEM allocation, and one thread that issues tcgen05.mma (M=128, N=TM, K=16, A from
//            TMEM, B from shared memory) x 8 per stage into the f32 accumulator (TM columns);
//            tcgen05.commit frees the shared-memory stage and the TMEM slot.
//   warps 2-17 then run the epilogue: tcgen05.ld of their lanes (one weight row, consecutive
//            activation rows), bias, conversion into a [TM][128] tile in the idle stage buffers,
//            then 16-byte stores of whole Y row segments.
// The shared-memory ring (2-4 stages) and the TMEM slot ring (4) are independent, so the copies,
// the dequantisation and the MMAs overlap instead of paying their latencies in sequence.
// Every mbarrier wait is bounded by a clock deadline; a wait that runs out writes the device
// status word, raises the CTA's abort flag and the CTA winds down (no trap, no endless spin).
#include "internal.cuh"
#include "sm100.cuh"

#include <map>
#include <memory>
#include <mutex>

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

// The pairs (e0, e1) and (e2, e3) of stage position j (k = 16j + 4tp + e) as O + q in the MMA
// type, O = 1024 (f16) or 128 (bf16), for 2- and 8-bit weights (4-bit: q_pairs4 and the fused
// path). `x` is the packed word holding position j and `sh` the shift of its pair within it, in
// packed_position's order: 8 bits, byte e of the word; 2 bits, bits 4jj + 16(e & 1) + 2(e >> 1)
// for jj = j mod 4. 8-bit weights only in f16 (128 + q is not exact in bf16 from q = 128).
template <int BITS, bool BF>
__device__ __forceinline__ void magic_pairs(uint32_t x, int sh, uint32_t& pa, uint32_t& pb) {
  constexpr uint32_t M = BF ? 0x43004300u : 0x64006400u;
  if constexpr (BITS == 8) {
    static_assert(!BF, "8-bit magic pairs are f16 only");
    pa = __byte_perm(x, 0x64646464u, 0x4140);  // bytes 0, 1 under the f16 exponent of 1024
    pb = __byte_perm(x, 0x64646464u, 0x4342);
  } else {
    static_assert(BITS == 2, "4-bit weights take q_pairs4");
    const uint32_t src = x >> sh;
    pa = lop3_and_or(src, 0x00030003u, M);
    pb = lop3_and_or(src >> 2, 0x00030003u, M);
  }
}

// q of the pairs (e0, e1) and (e2, e3) as exact values of the MMA type (2- and 8-bit weights).
template <int BITS, bool BF>
__device__ __forceinline__ void exact_pairs(uint32_t x, int sh, uint32_t& q0, uint32_t& q1) {
  if constexpr (BITS == 8 && BF) {  // q <= 255: exact in bf16
    __nv_bfloat162 a = __floats2bfloat162_rn((float)(x & 0xFFu), (float)((x >> 8) & 0xFFu));
    __nv_bfloat162 b = __floats2bfloat162_rn((float)((x >> 16) & 0xFFu), (float)(x >> 24));
    q0 = *reinterpret_cast<uint32_t*>(&a);
    q1 = *reinterpret_cast<uint32_t*>(&b);
  } else {
    constexpr uint32_t M = BF ? 0x43004300u : 0x64006400u;
    uint32_t pa, pb;
    magic_pairs<BITS, BF>(x, sh, pa, pb);
    q0 = h2_sub(pa, M, BF);
    q1 = h2_sub(pb, M, BF);
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

// 2 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st2(uint32_t taddr, uint32_t r0, uint32_t r1) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1,%2};" ::"r"(taddr), "r"(r0), "r"(r1) : "memory");
}

// 8 consecutive 32-bit TMEM columns of this thread's lane (loaded and waited for).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct GemmArgs {
  float z_const;
  int has_zp;
  int bs_log2;
  int nb;          // scale blocks per stage (the TMA box height)
  int M, N, K;
  int ktiles;      // 128-k stages per row
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
  const float* row_scale;  // per activation row factor of an f32 A carried as scaled f16, or null
  const int32_t* wexp;     // per weight row exponent of f32 weights carried as scaled f16 / bf16, or null
  int ks;                  // CTAs splitting K in a cluster (1: none)
  int s16;                 // f32 weights with the handle's f16 block scales (scales16): packed dequant
};

constexpr int kDeqWarps = 16;      // dequantising / epilogue warps: 4 per TMEM lane quarter
constexpr int kGemmThreads = 64 + 32 * kDeqWarps;  // + the producer and MMA warps
constexpr int WN = 128;            // weight rows per CTA: the MMA's M and the TMEM lanes
constexpr int kMaxStages = 8;      // shared-memory stages
constexpr int kASlots = 4;         // dequantised weight stages in TMEM, 64 columns each (at most)
constexpr int kSmemSM = 233472;    // shared memory of an SM

// A stage covers 128 k: the packed weights of one 64-byte group for 4 bits, two groups for 8
// bits, and for 2 bits the group of 256 k whose half the stage uses (the group is loaded whole).
template <int TM, int BITS>
struct GemmTile {
  static constexpr int ACT_BYTES = TM * 128 * 2;  // TM rows x 128 k x 2 B (two SW128 halves)
  static constexpr int WP_BYTES = WN * (BITS == 8 ? 128 : 64);  // packed
  static constexpr int FIXED = ACT_BYTES + WP_BYTES;
  static_assert(TM % 32 == 0 && TM >= 32 && TM <= 256, "MMA N");
  // Tiles of at most 64 activation rows: 3 weight slots in 256 TMEM columns, two CTAs per SM (the
  // second CTA's start-up and epilogue overlap the first's work); wider tiles: 4 slots, all 512
  // columns, one CTA per SM.
  static constexpr int SLOTS = TM <= 64 ? 3 : 4;
  static constexpr int COLS = TM <= 64 ? 256 : 512;
  static constexpr int CTAS = TM <= 64 ? 2 : 1;
  // Dequantising teams: up to 128 activation rows the MMAs of a stage are short and a stage took
  // one warp's chain of latencies (waits, shared-memory loads, TMEM stores, tcgen05.wait::st)
  // with all 16 warps on it; two teams of 8 on alternate stages, each warp converting two pieces
  // of its row, overlap those chains (C2 11.3 -> 10.2 us, C3 M = 64 89.7 -> 75.8 us, C5 M = 16
  // 37.6 -> 35.4 us). With 256 rows the MMAs bound the stage and one team measured 1-2% faster.
  static constexpr int TEAMS = TM <= 128 ? 2 : 1;
  static constexpr int PIECES = TEAMS;  // 16-byte pieces of its row a warp converts per stage
  static_assert(TM + SLOTS * 64 <= COLS && SLOTS <= kASlots, "TMEM columns");
};

// HOIST: block_size >= 128, so one block covers each 128-k stage and its scale and zero point are
// read once per stage instead of per position.
template <int TM, bool BF, tq4_dtype T, int BITS, bool HOIST>
__global__ void __launch_bounds__(kGemmThreads, GemmTile<TM, BITS>::CTAS)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_z,
                const GemmArgs p) {
  using L = GemmTile<TM, BITS>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const int S = p.stages;
  const uint32_t bars = base + S * p.stage_bytes;
  auto full = [&](int s) { return bars + 8 * s; };                        // activations landed
  auto empty = [&](int s) { return bars + 8 * (kMaxStages + s); };
  auto afull = [&](int a) { return bars + 8 * (2 * kMaxStages + a); };
  auto aempty = [&](int a) { return bars + 8 * (2 * kMaxStages + kASlots + a); };
  const uint32_t accum = bars + 8 * (2 * kMaxStages + 2 * kASlots);
  auto wfull = [&](int s) { return bars + 8 * (2 * kMaxStages + 2 * kASlots + 1 + s); };  // weights landed
  uint8_t* tail = smem + S * p.stage_bytes + 8 * (3 * kMaxStages + 2 * kASlots + 1);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(tail);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tail + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Split K: the ks CTAs of a cluster (consecutive along x) take consecutive k-tile ranges.
  int kr = 0, n0 = blockIdx.x * WN, kt0 = 0, KT = p.ktiles;  // this CTA's k-tiles: [kt0, kt0 + KT)
  const int m0 = blockIdx.y * TM;
  if (p.ks > 1) {
    kr = blockIdx.x % p.ks;
    n0 = (blockIdx.x / p.ks) * WN;
    kt0 = p.ktiles * kr / p.ks;
    KT = p.ktiles * (kr + 1) / p.ks - kt0;
  }
  const uint32_t tx_a = L::ACT_BYTES;
  const uint32_t tx_w = L::WP_BYTES + WN * p.nb * p.st_bytes * (p.has_zp ? 2 : 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(wfull(s), 1);
      mbar_init(empty(s), 1 + kDeqWarps / L::TEAMS);  // the MMAs' commit + the stage's team
    }
    for (int a = 0; a < L::SLOTS; ++a) {
      mbar_init(afull(a), kDeqWarps / L::TEAMS);
      mbar_init(aempty(a), 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)tmem_slot)), "r"((uint32_t)L::COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;
  // The next kernel on the stream may be scheduled only once this CTA holds its tensor memory:
  // a dependent CTA that took an SM's TMEM first would block this CTA's allocation while it
  // waits for this grid (and a GEMM CTA owns its SM's shared memory, see plan_gemm_smem).
  pdl_trigger();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // The packed weights of stage kt (absolute): 64-byte groups of 512 / BITS k each.
      auto load_w = [&](uint32_t st, int kt, uint32_t bar) {
        if constexpr (BITS == 8) {
          tma_load_2d(st + L::ACT_BYTES, &map_w, kt * 128, n0, bar);
          tma_load_2d(st + L::ACT_BYTES + WN * 64, &map_w, kt * 128 + 64, n0, bar);
        } else if constexpr (BITS == 2) {
          tma_load_2d(st + L::ACT_BYTES, &map_w, (kt >> 1) * 64, n0, bar);
        } else {
          tma_load_2d(st + L::ACT_BYTES, &map_w, kt * 64, n0, bar);
        }
      };
      // The first ring's weights, scales and zero points are constant: they load before the
      // previous kernel on the stream has finished (programmatic dependent launch); the
      // activations of those stages follow once it has.
      const int pre = min(S, KT);
      for (int kt = 0; kt < pre; ++kt) {
        const uint32_t st = base + kt * p.stage_bytes;
        const int b0 = ((kt0 + kt) * 128) >> p.bs_log2;
        mbar_expect_tx(wfull(kt), tx_w);
        load_w(st, kt0 + kt, wfull(kt));
        tma_load_2d(st + p.sc_off, &map_s, n0, b0, wfull(kt));
        if (p.has_zp) tma_load_2d(st + p.zc_off, &map_z, n0, b0, wfull(kt));
      }
      pdl_wait();
      for (int kt = 0; kt < pre; ++kt) {
        const uint32_t st = base + kt * p.stage_bytes;
        mbar_expect_tx(full(kt), tx_a);
        tma_load_2d(st, &map_a, (kt0 + kt) * 128, m0, full(kt));
        tma_load_2d(st + L::ACT_BYTES / 2, &map_a, (kt0 + kt) * 128 + 64, m0, full(kt));
      }
      int issued = pre;
      for (int kt = pre; kt < KT; ++kt) {
        const int s = kt % S;
        const uint32_t ph = (kt / S) & 1;
        if (!mbar_wait(empty(s), ph ^ 1, abort_flag, kDevTimeoutStageEmpty)) break;
        const uint32_t st = base + s * p.stage_bytes;
        const int b0 = ((kt0 + kt) * 128) >> p.bs_log2;
        mbar_expect_tx(wfull(s), tx_w);
        load_w(st, kt0 + kt, wfull(s));
        tma_load_2d(st + p.sc_off, &map_s, n0, b0, wfull(s));
        if (p.has_zp) tma_load_2d(st + p.zc_off, &map_z, n0, b0, wfull(s));
        mbar_expect_tx(full(s), tx_a);
        tma_load_2d(st, &map_a, (kt0 + kt) * 128, m0, full(s));
        tma_load_2d(st + L::ACT_BYTES / 2, &map_a, (kt0 + kt) * 128 + 64, m0, full(s));
        issued = kt + 1;
      }
      // the copies still in flight complete before the CTA exits (bounded)
      for (int kt = max(0, issued - S); kt < issued; ++kt) {
        mbar_drain(full(kt % S), (kt / S) & 1);
        mbar_drain(wfull(kt % S), (kt / S) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | ((BF ? 1u : 0u) << 7) | ((BF ? 1u : 0u) << 10) |
                                 ((uint32_t)(TM >> 3) << 17) | ((uint32_t)(WN >> 4) << 24);
      bool ok = true;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int s = kt % S, a = kt % L::SLOTS;
        ok = mbar_wait(full(s), (kt / S) & 1, abort_flag, kDevTimeoutTmaFull) &&
             mbar_wait(afull(a), (kt / L::SLOTS) & 1, abort_flag, kDevTimeoutDequant);
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
    const int tp = (warp - 2) >> 2;        // 16-byte piece tp of its row: k = 16j + 4tp + e, j = 0..7
    const int r = quarter * 32 + lane;     // this thread's weight row in the tile
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    constexpr bool T_SAME = (BF && T == TQ4_BF16) || (!BF && T == TQ4_F16);
    const int we = (T == TQ4_F32 && p.wexp) ? p.wexp[n0 + r] : 0;  // n0 + r < n_pad
    // 2^we and 2^-we once per thread: multiplying by them rounds exactly like ldexpf while both
    // are normal numbers; ldexpf itself for the rare rows outside that range
    const bool pw_ok = we > -126 && we < 126;
    const float pw_up = ldexpf(1.f, we), pw_down = ldexpf(1.f, -we);
    constexpr bool kFusedOk = !(BF && BITS == 8);
    // the packed f16 / bf16 path: exact (O + q) - (O + z), then one multiply (uniform for the call)
    const bool fused = kFusedOk && (T_SAME || (T == TQ4_F32 && p.s16)) && p.int_zp;
    // L::TEAMS teams take alternate stages; with two, team (warp - 2) / 8 converts pieces 2 tpt
    // and 2 tpt + 1 of each of its rows (GemmTile::TEAMS)
    constexpr int PIECES = L::PIECES;
    const int team = (warp - 2) / (kDeqWarps / L::TEAMS);
    const int tpt = L::TEAMS == 2 ? ((warp - 2) >> 2) & 1 : tp;  // the warp's piece pair (or piece)
    for (int kt = team; kt < KT; kt += L::TEAMS) {
      const int s = kt % S, a = kt % L::SLOTS;
      if (!mbar_wait(wfull(s), (kt / S) & 1, abort_flag, kDevTimeoutTmaFull)) break;
      if (!mbar_wait(aempty(a), ((kt / L::SLOTS) & 1) ^ 1, abort_flag, kDevTimeoutDequant)) break;
      const uint8_t* st = smem + s * p.stage_bytes;
      // the 64-byte swizzle puts piece q of row r at 16 * (q ^ ((r >> 1) & 3)): the 8 lanes of
      // each load phase read 8 different bank groups
      uint4 vp[PIECES], vp1[PIECES];
#pragma unroll
      for (int pi = 0; pi < PIECES; ++pi) {
        const int q = PIECES * tpt + pi;
        const uint32_t piece = r * 64 + ((q ^ ((r >> 1) & 3)) << 4);
        vp[pi] = *reinterpret_cast<const uint4*>(st + L::ACT_BYTES + piece);
        // 8 bits: the stage's second group (positions j = 4..7); 2 bits: which half of the group
        vp1[pi] = BITS == 8 ? *reinterpret_cast<const uint4*>(st + L::ACT_BYTES + WN * 64 + piece) : vp[pi];
      }
      const int half = (kt0 + kt) & 1;
      const uint8_t* sc = st + p.sc_off;
      const uint8_t* zc = st + p.zc_off;
      const int b0 = ((kt0 + kt) * 128) >> p.bs_log2;
      // column 8j + 2q holds k = 16j + 4q, +1 (piece q)
      const uint32_t col0 = lane_addr + TM + a * 64 + 2 * PIECES * tpt;
      uint32_t s2 = 0, oz2 = 0, oz16n = 0;
      float scv = 0.f, z = 0.f;
      auto block_params = [&](int lb) {  // the scale and zero point of staged block row lb
        if (fused) {
          const uint32_t sv = reinterpret_cast<const uint16_t*>(sc)[lb * WN + r];
          s2 = sv | (sv << 16);
          z = p.has_zp ? scale_to_f32(zc, lb * WN + r, 2, BF) : p.z_const;
          oz2 = h2_splat((BF ? 128.f : 1024.f) + z, BF);
          oz16n = h2_splat(-(64.f + z), BF);
        } else {
          const float sraw = scale_to_f32(sc, lb * WN + r, p.st_bytes, T == TQ4_BF16);
          scv = pw_ok ? sraw * pw_down : ldexpf(sraw, -we);
          z = p.has_zp ? scale_to_f32(zc, lb * WN + r, p.st_bytes, T == TQ4_BF16) : p.z_const;
        }
      };
      if constexpr (HOIST) block_params(0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if constexpr (!HOIST) {
          const int lb = (((kt0 + kt) * 128 + 16 * j) >> p.bs_log2) - b0;  // staged block row
          if ((j == 0) || (((16 * j) & ((1 << p.bs_log2) - 1)) == 0)) block_params(lb);
        }
#pragma unroll
        for (int pi = 0; pi < PIECES; ++pi) {
          const uint4& v = vp[pi];
          const uint4& v1 = vp1[pi];
          uint32_t x;
          int sh = 0;
          if constexpr (BITS == 4) {
            x = (j < 2) ? v.x : (j < 4) ? v.y : (j < 6) ? v.z : v.w;
          } else if constexpr (BITS == 8) {
            const uint4& vv = j < 4 ? v : v1;
            x = ((j & 3) == 0) ? vv.x : ((j & 3) == 1) ? vv.y : ((j & 3) == 2) ? vv.z : vv.w;
          } else {
            x = half ? ((j < 4) ? v.z : v.w) : ((j < 4) ? v.x : v.y);
            sh = 4 * (j & 3);
          }
          uint32_t w0, w1;
          if (fused) {
            // (O + q) - (O + z) is exact in the MMA type; one more multiply gives RN_T((q - z) * s)
            // (f32 weights: times the f16 s * 2^-we of the handle's scales16)
            const uint32_t src = (j & 1) ? (x >> 8) : x;
            uint32_t d0, d1;
            if constexpr (BITS != 4 && kFusedOk) {
              uint32_t pa, pb;
              magic_pairs<BITS, BF>(x, sh, pa, pb);
              d0 = h2_sub(pa, oz2, BF);
              d1 = h2_sub(pb, oz2, BF);
            } else if (!BF) {
              d0 = h2_sub(lop3_and_or(src, 0x000F000Fu, 0x64006400u), oz2, false);
              const uint32_t r1 = lop3_and_or(src, 0x00F000F0u, 0x64006400u);  // 1024 + 16 q
              asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d1) : "r"(r1), "r"(0x2C002C00u), "r"(oz16n));
            } else {
              d0 = h2_sub(lop3_and_or(src, 0x000F000Fu, 0x43004300u), oz2, true);
              d1 = h2_sub(lop3_and_or(src >> 4, 0x000F000Fu, 0x43004300u), oz2, true);
            }
            w0 = h2_mul(d0, s2, BF);
            w1 = h2_mul(d1, s2, BF);
          } else {
            // f32 weights: (q - z) * s * 2^-we, exact scaling of the f32 product before its rounding
            uint32_t q0, q1;
            if constexpr (BITS == 4) q_pairs4(x, j, BF, q0, q1);
            else exact_pairs<BITS, BF>(x, sh, q0, q1);
            w0 = deq_pair<BF, T>(q0, z, scv);
            w1 = deq_pair<BF, T>(q1, z, scv);
          }
          tmem_st2(col0 + 8 * j + 2 * pi, w0, w1);
        }
      }
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
    while (!mbar_test(accum, 0)) {
      if (clock64() - t0 > wait_limit()) {
        report(kDevTimeoutAccum);
        *abort_flag = 1;
        ok = false;
        break;
      }
    }
    asm volatile("tcgen05.fence::after_thread_sync;");
    // D (TMEM lane = weight row, column = activation row) -> the tile [TM][128] in Y's type in the
    // now idle stage buffers -> coalesced 16-byte stores of Y rows.
    const int ys = p.y_t == TQ4_F32 ? 4 : 2;
    const int64_t n = (int64_t)n0 + r;
    const bool n_ok = n < p.N;
    const float bias_v = (p.bias && n_ok) ? load_as_f32(p.bias, n, p.bias_t) : 0.f;
    const bool run = __all_sync(0xffffffffu, ok && !*abort_flag);
    constexpr int CPW = TM / 4;  // activation rows (TMEM columns) per warp
    if (run && p.ks > 1) {  // split K: this CTA's raw sums, [TM][128] f32, for the cluster to add
#pragma unroll 1
      for (int c = tp * CPW; c < (tp + 1) * CPW; c += 8) {
        uint32_t rr[8];
        tmem_ld8(lane_addr + c, rr);
#pragma unroll
        for (int i = 0; i < 8; ++i) reinterpret_cast<float*>(smem)[(c + i) * WN + r] = __uint_as_float(rr[i]);
      }
    } else if (run) {
#pragma unroll 1
      for (int c = tp * CPW; c < (tp + 1) * CPW; c += 8) {
        uint32_t rr[8];
        tmem_ld8(lane_addr + c, rr);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int ml = c + i;
          float v = __uint_as_float(rr[i]);
          if (we) v = pw_ok ? v * pw_up : ldexpf(v, we);
          if (p.row_scale && m0 + ml < p.M) v *= p.row_scale[m0 + ml];  // a power of two: exact
          if (p.bias) v = round_to(v, p.y_t) + bias_v;
          uint8_t* dst = smem + ((int64_t)ml * WN + r) * ys;
          if (p.y_t == TQ4_F32) *reinterpret_cast<float*>(dst) = v;
          else if (p.y_t == TQ4_BF16) *reinterpret_cast<__nv_bfloat16*>(dst) = __float2bfloat16_rn(v);
          else *reinterpret_cast<__half*>(dst) = __float2half_rn(v);
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kDeqWarps) : "memory");
    if (run && p.ks == 1) {
      const int rows = min(TM, p.M - m0);
      const int cpr = WN * ys / 16;  // 16-byte chunks per tile row
      const int epc = 16 / ys;       // elements per chunk
      const int tid = threadIdx.x - 64;
      for (int i = tid; i < rows * cpr; i += 32 * kDeqWarps) {
        const int ml = i / cpr, cc = i % cpr;
        const int64_t nn = (int64_t)n0 + cc * epc;
        const uint8_t* src = smem + ((int64_t)ml * WN + cc * epc) * ys;
        uint8_t* dst = static_cast<uint8_t*>(p.y) + ((int64_t)(m0 + ml) * p.ldy + nn) * ys;
        if (nn + epc <= p.N && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
          *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
        } else {
          for (int e = 0; e < epc && nn + e < p.N; ++e)
            for (int b = 0; b < ys; ++b) dst[e * ys + b] = src[e * ys + b];
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
  }

  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)L::COLS));
  }
  if (p.ks > 1) {
    // Every CTA of the cluster has its raw [TM][128] sums in shared memory. Rank kr adds the
    // ranks' sums of activation rows [kr TM / ks, (kr + 1) TM / ks) in rank order (the result
    // does not depend on scheduling), finishes them like the single-CTA epilogue (weight-row
    // exponent, activation-row scale, bias) and stores Y. The second barrier keeps every CTA's
    // shared memory alive until all ranks have read it.
    cluster_sync_all();
    const float* part = reinterpret_cast<const float*>(smem);
    const int rows = min(TM, p.M - m0);
    const int r_lo = kr * TM / p.ks, r_hi = min(rows, (kr + 1) * TM / p.ks);
    const int units = max(0, r_hi - r_lo) * (WN / 4);
    for (int i = threadIdx.x; i < units; i += kGemmThreads) {
      const int ml = r_lo + i / (WN / 4), c = (i % (WN / 4)) * 4;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      for (int q = 0; q < p.ks; ++q) {
        const float4 x = ld_cluster_f32x4(part + ml * WN + c, (unsigned)q);
        v[0] += x.x;
        v[1] += x.y;
        v[2] += x.z;
        v[3] += x.w;
      }
      const float rs = p.row_scale ? p.row_scale[m0 + ml] : 1.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t n = (int64_t)n0 + c + e;
        if (n >= p.N) break;
        float y = v[e];
        if (T == TQ4_F32 && p.wexp) y = ldexpf(y, p.wexp[n]);
        y *= rs;  // a power of two: exact
        if (p.bias) y = round_to(y, p.y_t) + load_as_f32(p.bias, n, p.bias_t);
        store_from_f32(p.y, (int64_t)(m0 + ml) * p.ldy + n, p.y_t, y);
      }
    }
    cluster_sync_all();
  }
}

// f32 activations for the tensor cores: row m of A becomes f16 values a * 2^-e(m), e(m) the
// exponent of the row's largest magnitude (so every value is at most 2 and none overflows), and
// row_scale[m] = 2^e(m) is multiplied back in the epilogue. The rounding to f16 is the only
// change to A (relative 2^-11, like the GEMV's staged activations).
__global__ void __launch_bounds__(256) scale_rows_f16_kernel(const float* __restrict__ a, int64_t k,
                                                             __half* __restrict__ out, float* __restrict__ row_scale) {
  __shared__ float red[8];
  const float* row = a + blockIdx.x * k;
  float mx = 0.f;
  for (int64_t i = threadIdx.x; i < k; i += 256) mx = fmaxf(mx, fabsf(row[i]));
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  int e = 0;
  if (mx > 0.f && isfinite(mx)) frexpf(mx, &e);  // mx = f * 2^e, f in [0.5, 1)
  const float down = ldexpf(1.f, -e);
  for (int64_t i = threadIdx.x; i < k; i += 256) out[blockIdx.x * k + i] = __float2half_rn(row[i] * down);
  if (threadIdx.x == 0) row_scale[blockIdx.x] = ldexpf(1.f, e);
}

// Per-(device, stream) scratch of the scaled f16 activations.
struct RowScratch {
  DeviceBuffer a16, scale;
};
static std::mutex g_row_mu;
static std::map<std::pair<int, cudaStream_t>, std::unique_ptr<RowScratch>> g_row_scratch;

static tq4_status row_scratch(cudaStream_t st, int64_t a_bytes, int64_t rows, void** a16, float** scale) {
  int dev = 0;
  TQ4_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_row_mu);
  auto& slot = g_row_scratch[{dev, st}];
  if (!slot) slot.reset(new RowScratch());
  if (slot->a16.bytes < a_bytes || slot->scale.bytes < rows * 4) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    TQ4_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone) {
      set_error("MatMulNBits: an f32 prefill call needs scratch first allocated during stream capture; "
                "make the same call once before capturing");
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    TQ4_CUDA(cudaStreamSynchronize(st));
    if (slot->a16.bytes < a_bytes) TQ4_TRY(slot->a16.alloc(a_bytes));
    if (slot->scale.bytes < rows * 4) TQ4_TRY(slot->scale.alloc(rows * 4));
  }
  *a16 = slot->a16.ptr;
  *scale = static_cast<float*>(slot->scale.ptr);
  return TQ4_OK;
}

// ---- host side ---------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  // looked up once per process (a function-local static: thread-safe initialisation)
  static const EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return nullptr;
  }();
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

// Descriptors of a new handle: the packed rows (box 128 rows x one 64-byte group, whatever the bit
// width) and the block-major scales / zero points (box 128 rows x the stage's blocks).
tq4_status make_weight_maps(Weight& w) {
  w.wmaps_ok = false;
  if (encode_fn() == nullptr) return TQ4_OK;
  const int st = dtype_size(w.desc.dequant_dtype);
  const CUtensorMapDataType sdt = st == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const int nb = gemm_scale_blocks(w);
  TQ4_TRY(make_map(&w.wmaps[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q.ptr, w.row_bytes, w.n_pad, w.row_bytes, 64,
                   WN, CU_TENSOR_MAP_SWIZZLE_64B));  // 16-byte piece c of row r at c ^ ((r >> 1) & 3)
  TQ4_TRY(make_map(&w.smaps[0], sdt, w.scales.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, WN, nb,
                   CU_TENSOR_MAP_SWIZZLE_NONE));
  if (w.zps.ptr)
    TQ4_TRY(make_map(&w.zmaps[0], sdt, w.zps.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, WN, nb,
                     CU_TENSOR_MAP_SWIZZLE_NONE));
  else
    w.zmaps[0] = w.smaps[0];  // never loaded
  w.s16_ok = false;
  if (w.scales16.ptr) {
    TQ4_TRY(make_map(&w.smap16, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.scales16.ptr, w.n_pad, w.blocks_pad, w.n_pad * 2, WN,
                     nb, CU_TENSOR_MAP_SWIZZLE_NONE));
    w.s16_ok = true;
  }
  w.wmaps_ok = true;
  return TQ4_OK;
}

constexpr int kSmemLimit = 232448;  // 227 KB of dynamic shared memory per CTA

struct GemmPlan {
  int stages, stage_bytes, sc_off, zc_off, smem;
};

template <int TM, int BITS>
static GemmPlan plan_gemm_smem(const Weight& w, int st) {  // st: bytes of a staged scale
  using L = GemmTile<TM, BITS>;
  GemmPlan pl{};
  const int sc_bytes = WN * gemm_scale_blocks(w) * st;
  pl.sc_off = L::FIXED;
  pl.zc_off = pl.sc_off + (sc_bytes + 127) / 128 * 128;
  const int end = pl.zc_off + (w.zps.ptr ? sc_bytes : 0);
  pl.stage_bytes = (end + 1023) / 1024 * 1024;
  const int fixed = 1024 + 8 * (3 * kMaxStages + 2 * kASlots + 1) + 16;
  // L::CTAS GEMM CTAs per SM, and no more: a CTA that allocates tensor memory should never share
  // its SM with a CTA that could only sit blocked in its own allocation. Each CTA asks for more
  // than 1 / (CTAS + 1) of the SM's shared memory (the 1 KB per CTA the runtime keeps included).
  const int cap = L::CTAS == 1 ? kSmemLimit : kSmemSM / L::CTAS - 1024;
  pl.stages = std::min(kMaxStages, (cap - fixed) / pl.stage_bytes);
  pl.smem = fixed + pl.stages * pl.stage_bytes;
  pl.smem = std::max(pl.smem, kSmemSM / (L::CTAS + 1) + 1024);
  return pl;
}

using GemmKernel = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, GemmArgs);

// One launch of `kern` (its own once-per-device shared-memory attribute flag in `attr_set`).
static tq4_status launch_gemm_kern(GemmKernel kern, std::atomic<uint64_t>& attr_set, const GemmPlan& pl, int tm,
                                   const CUtensorMap& ma, const Weight& w, const GemmArgs& args, cudaStream_t st) {
  TQ4_CUDA(set_smem_limit_once(kern, kSmemLimit, attr_set));
  const dim3 grid(((args.N + WN - 1) / WN) * args.ks, (args.M + tm - 1) / tm);
  if (args.ks == 1) {
    TQ4_CUDA(launch_pdl(kern, grid, dim3(kGemmThreads), pl.smem, st, ma, w.wmaps[0], args.s16 ? w.smap16 : w.smaps[0],
                        w.zmaps[0], args));
    return TQ4_OK;
  }
  // split K: a cluster of ks CTAs along x, plus the dependent launch
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = args.ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  TQ4_CUDA(cudaLaunchKernelEx(&cfg, kern, ma, w.wmaps[0], args.s16 ? w.smap16 : w.smaps[0], w.zmaps[0], args));
  return TQ4_OK;
}

template <int TM, bool BF, tq4_dtype T, int BITS>
static tq4_status launch_gemm_t(const CUtensorMap& ma, const Weight& w, GemmArgs args, cudaStream_t st) {
  const GemmPlan pl = plan_gemm_smem<TM, BITS>(w, args.st_bytes);
  if (pl.stages < 2) {
    set_error("GEMM: the stage does not fit shared memory");
    return TQ4_ERR_UNSUPPORTED;
  }
  args.stages = pl.stages;
  args.stage_bytes = pl.stage_bytes;
  args.sc_off = pl.sc_off;
  args.zc_off = pl.zc_off;
  if constexpr (BITS == 4) {
    if (w.bs_log2 >= 7) {  // one block per 128-k stage (the instantiation is kept to 4-bit weights)
      static std::atomic<uint64_t> attr_hoist{0};
      return launch_gemm_kern(gemm_kernel<TM, BF, T, BITS, true>, attr_hoist, pl, TM, ma, w, args, st);
    }
  }
  static std::atomic<uint64_t> attr_set{0};  // per device, at the largest size it can ask for
  return launch_gemm_kern(gemm_kernel<TM, BF, T, BITS, false>, attr_set, pl, TM, ma, w, args, st);
}

template <int TM, bool BF, int BITS>
static tq4_status launch_gemm_b(const CUtensorMap& ma, const Weight& w, const GemmArgs& args, cudaStream_t st) {
  switch (w.desc.dequant_dtype) {
    case TQ4_F16: return launch_gemm_t<TM, BF, TQ4_F16, BITS>(ma, w, args, st);
    case TQ4_BF16: return launch_gemm_t<TM, BF, TQ4_BF16, BITS>(ma, w, args, st);
    default: return launch_gemm_t<TM, BF, TQ4_F32, BITS>(ma, w, args, st);
  }
}

template <int TM, bool BF>
static tq4_status launch_gemm_tm(const CUtensorMap& ma, const Weight& w, const GemmArgs& args, cudaStream_t st) {
  switch (w.desc.bits) {
    case 2: return launch_gemm_b<TM, BF, 2>(ma, w, args, st);
    case 8: return launch_gemm_b<TM, BF, 8>(ma, w, args, st);
    default: return launch_gemm_b<TM, BF, 4>(ma, w, args, st);
  }
}

// 128-k stages per row (the k-tiles of the GEMM), whatever the bit width.
static int gemm_ktiles(const Weight& w) { return (int)((w.k_pad + 127) / 128); }

// Whether the tcgen05 GEMM takes this call (else A goes through the GEMV in 16-row slices).
static bool gemm_eligible(const Weight& w, const void* a, tq4_dtype a_t) {
  if (w.desc.bits != 2 && w.desc.bits != 4 && w.desc.bits != 8) return false;
  if (a_t != TQ4_F16 && a_t != TQ4_BF16 && a_t != TQ4_F32) return false;
  if ((w.desc.K * 2) % 16 != 0) return false;                    // TMA row stride
  if ((reinterpret_cast<uintptr_t>(a) & 15) != 0) return false;  // TMA base address
  return w.wmaps_ok;
}

// Activation rows per CTA: no wider than M needs, and the largest tile that still gives half the
// SMs a tile.
// When that leaves only a 64- or 32-row tile (each weight row dequantised again for every narrow
// activation tile), the widest tile with K split over a cluster of ks CTAs instead (ks a power
// of two up to 8, tiles x ks within one wave, at least 4 k-tiles per CTA); 32-row tiles (M <= 32)
// split K the same way when they leave most SMs idle.
static int choose_tm(const Weight& w, int64_t m, int* ks) {
  const int64_t nt = (w.desc.N + WN - 1) / WN;
  *ks = 1;
  int narrow = 32;
  for (int tm : {256, 128, 64}) {
    if (tm / 2 >= m) continue;  // the half-size tile already covers M
    if (((m + tm - 1) / tm) * nt >= w.num_sms / 2) {
      if (tm >= 128) return tm;
      narrow = tm;
      break;
    }
  }
  for (int tm : {256, 128, 64, 32}) {
    if (tm / 2 >= m && tm > 32) continue;
    const int64_t tiles = ((m + tm - 1) / tm) * nt;
    int k = 1;
    while (k < 8 && tiles * k * 2 <= w.num_sms && gemm_ktiles(w) / (k * 2) >= 4) k *= 2;
    if (k > 1) {
      *ks = k;
      return tm;
    }
  }
  return narrow;
}

tq4_status run_gemm_tc(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                       tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  const float* row_scale = nullptr;
  if (a_t == TQ4_F32) {  // carried as row-scaled f16 (scale_rows_f16_kernel)
    void* a16 = nullptr;
    float* rs = nullptr;
    TQ4_TRY(row_scratch(st, m * w.desc.K * 2, m, &a16, &rs));
    scale_rows_f16_kernel<<<(unsigned)m, 256, 0, st>>>(static_cast<const float*>(a), w.desc.K,
                                                       static_cast<__half*>(a16), rs);
    TQ4_CUDA(cudaGetLastError());
    a = a16;
    a_t = TQ4_F16;
    row_scale = rs;
  }
  int ks = 1;
  const int tm = choose_tm(w, m, &ks);
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
  args.ktiles = gemm_ktiles(w);
  args.st_bytes = dtype_size(w.desc.dequant_dtype);
  args.int_zp = w.desc.zp_kind != TQ4_ZP_FLOAT;
  args.bias = bias;
  args.bias_t = bias_t;
  args.y = y;
  args.y_t = y_t;
  args.ldy = ldy;
  args.row_scale = row_scale;
  args.wexp = static_cast<const int32_t*>(w.wexp.ptr);
  args.ks = ks;
  // f32 weights without zero points under f16 activations: the f16 block scales
  args.s16 = (w.s16_ok && a_t == TQ4_F16) ? 1 : 0;
  if (args.s16) args.st_bytes = 2;
  const bool bf = a_t == TQ4_BF16;
  switch (tm) {
    case 256: return bf ? launch_gemm_tm<256, true>(ma, w, args, st) : launch_gemm_tm<256, false>(ma, w, args, st);
    case 128: return bf ? launch_gemm_tm<128, true>(ma, w, args, st) : launch_gemm_tm<128, false>(ma, w, args, st);
    case 64: return bf ? launch_gemm_tm<64, true>(ma, w, args, st) : launch_gemm_tm<64, false>(ma, w, args, st);
    default: return bf ? launch_gemm_tm<32, true>(ma, w, args, st) : launch_gemm_tm<32, false>(ma, w, args, st);
  }
}

// Rows of A in slices of 16 through the fused GEMV kernel (A that TMA cannot address).
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
  // M <= 8: the fused GEMV. 9 <= M <= 16: the tensor-core GEMM on a 32-row activation tile when it
  // can take the call (measured on the C5 shapes at M = 16: 1.2-3x faster than the GEMV's two
  // 8-row column tiles), else the GEMV.
  if (m <= 8 || (m <= 16 && !gemm_eligible(w, a, a_t))) return run_gemv(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
  return run_gemm(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
}

}  // namespace tq4
