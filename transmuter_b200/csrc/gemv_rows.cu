// M = 1 MatMulNBits over 32-row units, for 4-bit weights: the 151936-column lm_head (C3), the
// K = 1024 decode projections, and (K-sliced) the longer rows of the Llama-shaped decode calls.
//
// Math: the MatMulNBits clause (quantized.ex:30-46) over dequantize_weight/4 (:234-240),
//   Y[n] = sum_k A[k] * (q[n][k] - z[n][b(k)]) * s[n][b(k)],
// with the weights entering mma.sync m16n8k16 as magic-number floats O + q/c(k) straight out of
// one LOP3 and the activations staged as v(k) = RN(A[k] / E * c(k)), E an exact power of two per
// segment (see gemv.cu for the derivation of the per-segment correction
//   Y[n] += s * (E * P - E * O * SV - z * E * SA)).
//
// Why 32-row units: the lm_head's 151936 rows are 1187 tiles of 128 rows. Handed out whole over
// 296 CTAs, the last 3 tiles make every call wait one more tile time at the end (4.01 tiles per
// CTA). 4748 units of 32 rows shrink that tail four-fold.
//
// Structure (persistent CTAs, kRowsCtas per SM; 8 consumer warps, a TMA producer warp and a reducer
// warp):
//   - A unit is 32 weight rows x the whole (padded) K: up to 8 boxes of 32 rows x 64 bytes of
//     packed weights, one per group, landing as [group][row][64 B] (rows 64 bytes apart: the
//     consumers' 16-byte loads are free of bank conflicts), plus one box of the block-major
//     scales (and zero points) of those rows: 32 rows x all blocks. One unit is one pipeline
//     stage. The weights are loaded with an L2 evict-first policy (read once per call).
//   - Consumer warp w always takes packed group w (k in [128w, 128w + 128)). So its 8 MMA B
//     fragments (the staged activations of its group; MMA column c holds segment c of the group,
//     the other columns see zero) and its segment factors are registers, built once per call by
//     warp shuffles from one 16-byte activation load per lane: no shared-memory staging, no
//     barrier between the warps before the first unit.
//   - Per unit, each consumer warp leaves its partial row sums in shared memory and arrives on
//     the stage's "partials" mbarrier; a reducer warp then frees the stage for the producer, adds
//     the groups' partials in group order (deterministic), applies the bias and stores the unit's
//     outputs (128-byte stores per destination). Keeping this work off the consumer warps keeps
//     them in step: a consumer that also reduced would fall behind and hold every stage longer.
//   - Units: CTA b first takes units b, b + G, ..., b + (S - 1) G (G CTAs, S stages), whose
//     copies are issued before the previous kernel on the stream has finished (programmatic
//     dependent launch: the weights are constant); the rest go out by ticket (an atomic counter)
//     in arrival order, so CTAs that stream faster take more (ticket arithmetic at the producer).
//   - Destinations: Y itself, or (N-sharded calls, sharded.cu) every rank's assembly buffer over
//     NVLink: the 32 outputs of a unit go to each destination with plain stores, into the half
//     that this call's epoch selects.
//   - Rows of more than 8 packed groups (K > 1024) run K-sliced: CTA b takes slice b % S of 8
//     groups for the whole call (so its warps' B fragments stay fixed), the slice's CTAs take its
//     units by their own ticket counter, and the reducer stores the slice's partial rows in a
//     workspace; rows_slice_sum_kernel then adds the slices in slice order (deterministic) and
//     applies the bias. (The cross-slice sum inside the reducer, with a fence and an arrival
//     counter per unit, held the consumers back and was slower than the 128-row kernel.)
// Every mbarrier wait is bounded; a wait that runs out writes the device status word and the CTA
// winds down.
#include "fragments.cuh"
#include "internal.cuh"
#include "rows.cuh"
#include "sm100.cuh"

namespace tq4 {

// Tuning constants (compile-time). Measured on the lm_head (C3, M = 1): 2 CTAs per SM and 32-row
// units are the fastest; 3 CTAs per SM (fewer stages each) and 64-row units were slower, and so
// were one contiguous bulk copy per unit instead of the per-group boxes, two units per ticket,
// and a grid smaller than the resident capacity.
#ifndef TQ4_ROWS_CTAS
#define TQ4_ROWS_CTAS 2  // CTAs per SM
#endif
#ifndef TQ4_ROWS_RU
#define TQ4_ROWS_RU 32  // weight rows per unit (32 or 64)
#endif

constexpr int kRU = TQ4_ROWS_RU;               // weight rows per unit
constexpr int kRB = kRU / 16;                  // MMA row blocks per unit
// Scale box rows: exactly the unit's rows. The correction loads of lanes t = 0 and 1 then meet in
// the same bank (2-way); 8 rows of padding would avoid that but re-read each neighbour's scales
// (measured 1% slower on C3).
constexpr int kSR = kRU;
static_assert(kRU == 32 || kRU == 64, "unit height");
constexpr int kRowsWarps = 8;                  // consumer warps: warp w takes group w
constexpr int kRowsProducer = kRowsWarps;      // the TMA producer warp
constexpr int kRowsReducer = kRowsWarps + 1;   // the warp that adds the groups' partials
constexpr int kRowsThreads = 32 * kRowsWarps + 64;
constexpr int kRowsMaxStages = 6;
constexpr int kRowsCtas = TQ4_ROWS_CTAS;
// Tail of the shared memory: full[], empty[] and pdone[] mbarriers, unit tags, abort flag.
constexpr int kRowsTail = 24 * kRowsMaxStages + 4 * kRowsMaxStages + 16;
// kRowsCtas CTAs per SM: each asks for at most its share of the SM's 228 KB, less the 1 KB the
// runtime keeps per CTA and 1 KB of alignment slack.
constexpr int kRowsSmemBudget = 233472 / kRowsCtas - 2048;

struct RowsArgs {
  const void* a;
  const void* bias;
  tq4_dtype bias_t;
  tq4_dtype y_t;
  void* y[kRowsMaxDst];  // destinations of Y (Y itself, or every rank's assembly buffer)
  int ndst;
  int64_t col0;                     // Y column of weight row 0
  const unsigned long long* epoch;  // sharded: this rank's completed-call count (null otherwise)
  int64_t half_elems;               // sharded: elements of one half of a destination buffer
  float z_const;
  int has_zp;
  int st_bytes, st_bf16;
  int K, N;
  int groups;
  int bs_log2;
  int nbs;  // scale blocks in a unit's box
  int units;
  int stages;
  int stage_bytes, sc_off, zc_off;
  int part_off, tail_off;
  int* counter;  // the units' tickets, one per K slice (zero between calls)
  const float* norm_w;  // RMSNorm weights of an f32 activation row (RowsNorm), or null
  float norm_eps;
  int slices;           // K slices of 8 packed groups (CTA b takes slice b % slices)
  float* ws;            // K-sliced: [slices][units * kRU] partial rows
};

template <tq4_dtype AT, int SPS>
__global__ void __launch_bounds__(kRowsThreads, kRowsCtas)
    gemv_rows_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_s,
                     const __grid_constant__ CUtensorMap map_z, const RowsArgs p) {
  constexpr bool BF = (AT == TQ4_BF16);
  // f32 activations take the precise weights (both pairs 1024 + 16 q) from 64-wide segments up,
  // as the 128-row kernel does
  constexpr bool PRECISE = (AT == TQ4_F32) && SPS > 2;
  constexpr int SEG = 16 * SPS;    // weights per segment (a block, or 128 of a longer block)
  constexpr int NSEG = 8 / SPS;    // segments per group: the MMA columns in use
  constexpr int LPS = SEG / 4;     // lanes per segment in the activation staging
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t sbase = (raw_addr + 1023) & ~1023u;  // TMA destinations 1024-byte aligned
  uint8_t* smem = smem_raw + (sbase - raw_addr);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  const uint32_t bars = sbase + p.tail_off;
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (kRowsMaxStages + s); };
  auto pdone = [&](int s) { return bars + 8 * (2 * kRowsMaxStages + s); };  // partials written
  uint8_t* tail = smem + p.tail_off;
  volatile int* tag = reinterpret_cast<volatile int*>(tail + 24 * kRowsMaxStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tail + 28 * kRowsMaxStages);
  float* part = reinterpret_cast<float*>(smem + p.part_off);  // [lap parity][stage][warp][kRU rows]
  // This CTA's K slice: packed groups [g0, g0 + sgroups), scale blocks from b0; the slice's CTAs
  // are numbered bi = 0 .. Gs - 1 (the grid is a multiple of the slice count).
  const int NS = p.slices, sl = blockIdx.x % NS, Gs = gridDim.x / NS, bi = blockIdx.x / NS;
  const int g0 = sl * kRowsWarps, sgroups = min(kRowsWarps, p.groups - g0);
  const int b0 = (g0 * 128) >> p.bs_log2;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);  // the reducer frees it once every consumer warp is done with it
      mbar_init(pdone(s), kRowsWarps);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kRowsProducer) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint32_t sc_bytes = (uint32_t)kSR * p.nbs * p.st_bytes;
      const uint32_t tx = (uint32_t)sgroups * kRU * 64 + sc_bytes * (p.has_zp ? 2u : 1u);
      const int G = Gs;  // the CTAs of this slice
      int* const counter = p.counter + sl;
      const int statics = S * G;
      // A unit's packed weights are read once per call: they leave L2 first, so the activations,
      // the outputs and the next kernel's inputs stay there (C3: 22.4 -> 21.4 us; the same hint on
      // the scales measured slower).
      const uint64_t pol_w = l2_evict_first_policy();
      // Ticket v hands out unit statics + v. Two tickets are kept in flight: an atomic's result is
      // used only a ticket later, so its round trip (long under a saturated memory system)
      // overlaps the waits for free stages. Tickets are used in the order they were taken, so when
      // one fails the one still in flight (taken after it) fails too: a CTA takes its successes
      // plus two failures, a call takes exactly (units - statics)+ + 2 G tickets, and the taker of
      // the last one puts the counter back to zero for the next call on the stream.
      const int succ = max(0, p.units - statics);
      const int tickets = succ + 2 * G;
      int s = 0, gs = 0;
      uint32_t ph = 0;
      auto advance = [&]() {
        ++gs;
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      };
      auto issue = [&](int u) {
        tag[s] = u;
        const uint32_t st = sbase + s * p.stage_bytes;
        mbar_expect_tx(full(s), tx);
        for (int gi = 0; gi < sgroups; ++gi)
          tma_load_2d_hint(st + gi * (kRU * 64), &map_w, (g0 + gi) * 64, u * kRU, full(s), pol_w);
        tma_load_2d(st + p.sc_off, &map_s, u * kRU, b0, full(s));
        if (p.has_zp) tma_load_2d(st + p.zc_off, &map_z, u * kRU, b0, full(s));
      };
      bool ok = true;
      // the static units: issued before the previous kernel on the stream has finished
      for (int i = 0; i < S && ok; ++i) {
        const int u = bi + i * G;
        if (u >= p.units) break;
        ok = mbar_wait(empty(s), ph ^ 1u, abort_flag, kDevTimeoutStageEmpty);
        if (ok) {
          issue(u);
          advance();
        }
      }
      pdl_wait();  // the ticket counter belongs to the stream's order
      // Runs ticket v's units; false once v fails (its partner then still has to be seen).
      auto run_ticket = [&](int v) {
        if (v == tickets - 1) *counter = 0;  // the call's last ticket
        if (v >= succ) return false;
        ok = mbar_wait(empty(s), ph ^ 1u, abort_flag, kDevTimeoutStageEmpty);
        if (ok) {
          issue(statics + v);
          advance();
        }
        return ok;
      };
      int qa = atomicAdd(counter, 1);
      int qb = atomicAdd(counter, 1);
      for (;;) {
        if (!run_ticket(qa)) {
          if (qb == tickets - 1) *counter = 0;
          break;
        }
        qa = atomicAdd(counter, 1);  // lands while qb's units are issued
        if (!run_ticket(qb)) {
          if (qa == tickets - 1) *counter = 0;
          break;
        }
        qb = atomicAdd(counter, 1);
      }
      // no work left: a stage that only says so
      if (ok && mbar_wait(empty(s), ph ^ 1u, abort_flag, kDevTimeoutStageEmpty)) {
        tag[s] = -1;
        mbar_arrive(full(s));
        advance();
      }
      // the copies still in flight land before the CTA exits (bounded)
      for (int g = max(0, gs - S); g < gs; ++g) mbar_drain(full(g % S), (g / S) & 1);
    }
    return;
  }

  if (warp == kRowsReducer) {
    // ---------------- reducer ----------------
    // Per unit: once every consumer warp has left its partials (pdone), free the stage for the
    // producer, then add the groups' partials in group order (deterministic), apply the bias and
    // store the unit's outputs to every destination. The partials are kept per lap parity: the
    // next lap of this stage writes the other half, and the lap after that cannot start before
    // this warp has freed the next lap's stage, which it does only after this reduction.
    pdl_wait();  // outputs belong to the stream's order
    const int64_t half = p.epoch ? (int64_t)(((*reinterpret_cast<const volatile unsigned long long*>(p.epoch)) + 1) & 1) *
                                       p.half_elems
                                 : 0;
    int s = 0;
    uint32_t ph = 0;
    for (;;) {
      if (!mbar_wait(full(s), ph, abort_flag, kDevTimeoutTmaFull)) break;
      const int u = tag[s];
      if (u < 0) break;  // the producer ran out of units
      if (!mbar_wait(pdone(s), ph, abort_flag, kDevTimeoutDequant)) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(s));
      const float* pr = part + (ph * S + s) * kRowsWarps * kRU;
      float vs[kRU / 32];
#pragma unroll
      for (int r = lane, i = 0; r < kRU; r += 32, ++i) {
        float v = 0.f;
        for (int w2 = 0; w2 < sgroups; ++w2) v += pr[w2 * kRU + r];
        vs[i] = v;
      }
      if (NS > 1) {
        // K-sliced: this slice's partial rows; rows_slice_sum_kernel adds the slices afterwards
        const int64_t n_ws = (int64_t)p.units * kRU;
#pragma unroll
        for (int r = lane, i = 0; r < kRU; r += 32, ++i) p.ws[sl * n_ws + (int64_t)u * kRU + r] = vs[i];
      } else {
#pragma unroll
        for (int r = lane, i = 0; r < kRU; r += 32, ++i) {
          float v = vs[i];
          const int64_t n = (int64_t)u * kRU + r;
          if (n < p.N) {
            if (p.bias) v = round_to(v, p.y_t) + load_as_f32(p.bias, n, p.bias_t);
            const int64_t off = half + p.col0 + n;
            for (int d = 0; d < p.ndst; ++d) store_from_f32(p.y[d], off, p.y_t, v);
          }
        }
      }
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const bool active = warp < sgroups;  // this warp's group: g0 + warp
  pdl_wait();  // the activations belong to the stream's order
  uint32_t bfr[8][2];
  float4 F[2];
  {
    // This warp's group of activations: lane L holds k = 128 (g0 + w) + 4 L .. + 3.
    float a4[4] = {0.f, 0.f, 0.f, 0.f};
    const int64_t k = (int64_t)(g0 + warp) * 128 + 4 * lane;
    if (active) load_act4<AT>(p.a, 0, k, p.K, (p.K & 3) == 0, a4);
    if (AT == TQ4_F32 && p.norm_w) {
      // RMSNorm prologue: the 8 consumer warps hold the whole row (groups * 128 >= K, zeros past
      // K); its mean square is summed in a fixed order, then a = (x * rs) * w.
      __shared__ float red[kRowsWarps];
      float ss = fmaf(a4[3], a4[3], fmaf(a4[2], a4[2], fmaf(a4[1], a4[1], a4[0] * a4[0])));
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) red[warp] = ss;
      asm volatile("bar.sync 1, %0;" ::"n"(kRowsWarps * 32) : "memory");
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kRowsWarps; ++i) tot += red[i];
      const float rs = 1.f / sqrtf(tot / (float)p.K + p.norm_eps);
#pragma unroll
      for (int e = 0; e < 4; ++e) a4[e] = (k + e < p.K) ? a4[e] * rs * p.norm_w[k + e] : 0.f;
    }
    float mx = fmaxf(fmaxf(fabsf(a4[0]), fabsf(a4[1])), fmaxf(fabsf(a4[2]), fabsf(a4[3])));
#pragma unroll
    for (int off = 1; off < LPS; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float e_scale = 1.f, inv = 1.f;
    if (mx > 0.f && mx <= 3.402823466e38f) {
      // mx = f * 2^ex with f in [0.5, 1): the segment is carried as a / 2^s with mx / 2^s in
      // [2^14, 2^15), so no staged value overflows f16 (or loses range in bf16)
      const int ex = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 126;
      const int sh = max(-126, min(127, ex - 15));
      e_scale = __uint_as_float((uint32_t)(sh + 127) << 23);
      inv = sh < 127 ? __uint_as_float((uint32_t)(127 - sh) << 23) : 5.8774717541e-39f;  // 2^-sh
    }
    uint32_t h[4];
    float sv = 0.f, sa = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float c = act_factor<4, BF, PRECISE>(e);  // 4 L is a multiple of 4
      const float c_inv = act_factor_inv<4, BF, PRECISE>(e);
      float val;
      if constexpr (BF) {
        const __nv_bfloat16 b = __float2bfloat16_rn(a4[e] * inv * c);
        h[e] = __bfloat16_as_ushort(b);
        val = __bfloat162float(b);
      } else {
        const __half b = __float2half_rn(a4[e] * inv * c);
        h[e] = __half_as_ushort(b);
        val = __half2float(b);
      }
      sv += val;
      sa += val * c_inv;  // exact: c is a power of two
    }
#pragma unroll
    for (int off = 1; off < LPS; off <<= 1) {
      sv += __shfl_xor_sync(0xffffffffu, sv, off);
      sa += __shfl_xor_sync(0xffffffffu, sa, off);
    }
    const uint32_t px = h[0] | (h[1] << 16), py = h[2] | (h[3] << 16);
    const float O = magic_offset<4, BF, PRECISE>();
    const float za = e_scale * sa;
    const float fx = e_scale * O * sv + (p.has_zp ? 0.f : p.z_const * za);
    // B fragment of step j (16 k): the lane 4 j + t run, in MMA column j / SPS only
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t x = __shfl_sync(0xffffffffu, px, 4 * j + t);
      const uint32_t y = __shfl_sync(0xffffffffu, py, 4 * j + t);
      const bool mine = (g == j / SPS);
      bfr[j][0] = mine ? x : 0u;
      bfr[j][1] = mine ? y : 0u;
    }
    // factors of the segments in this lane's accumulator columns 2t, 2t+1
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int sg = 2 * t + hh;
      const int src = (sg < NSEG ? sg : 0) * LPS;
      F[hh].x = __shfl_sync(0xffffffffu, e_scale, src);
      F[hh].y = __shfl_sync(0xffffffffu, fx, src);
      F[hh].z = __shfl_sync(0xffffffffu, za, src);
      F[hh].w = 0.f;
    }
  }

  int s = 0;
  uint32_t ph = 0;
  for (;;) {
    if (!mbar_wait(full(s), ph, abort_flag, kDevTimeoutTmaFull)) break;
    if (tag[s] < 0) break;  // the producer ran out of units
    const uint8_t* st = smem + s * p.stage_bytes;
    if (active) {
      const uint8_t* wt = st + warp * (kRU * 64);  // [group][row][64 B]
      const uint8_t* sc = st + p.sc_off;
      const uint8_t* zc = st + p.zc_off;
      float y[kRB][2];  // rows 16 rb + g and 16 rb + g + 8
#pragma unroll
      for (int rb = 0; rb < kRB; ++rb) y[rb][0] = y[rb][1] = 0.f;
#pragma unroll
      for (int rb = 0; rb < kRB; ++rb) {
        const uint4 xa = *reinterpret_cast<const uint4*>(wt + (rb * 16 + g) * 64 + t * 16);
        const uint4 xb = *reinterpret_cast<const uint4*>(wt + (rb * 16 + g + 8) * 64 + t * 16);
        float blk2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // even / odd steps
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t a0, a1, a2, a3;
          weight_pairs<4, BF, PRECISE>(word_of(xa, j / 2), j, a0, a2);
          weight_pairs<4, BF, PRECISE>(word_of(xb, j / 2), j, a1, a3);
          mma16816<BF>(blk2[j & 1], a0, a1, a2, a3, bfr[j][0], bfr[j][1]);
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int sg = 2 * t + hh;
          if (sg < NSEG) {
            const int lb = (((g0 + warp) * 128 + sg * SEG) >> p.bs_log2) - b0;  // its block in the box
            const int r0 = rb * 16 + g;
            const float s0 = scale_to_f32(sc, lb * kSR + r0, p.st_bytes, p.st_bf16);
            const float s8 = scale_to_f32(sc, lb * kSR + r0 + 8, p.st_bytes, p.st_bf16);
            float z0 = 0.f, z8 = 0.f;
            if (p.has_zp) {
              z0 = scale_to_f32(zc, lb * kSR + r0, p.st_bytes, p.st_bf16);
              z8 = scale_to_f32(zc, lb * kSR + r0 + 8, p.st_bytes, p.st_bf16);
            }
            const float d0 = blk2[0][hh] + blk2[1][hh], d8 = blk2[0][2 + hh] + blk2[1][2 + hh];
            y[rb][0] = fmaf(s0, fmaf(-z0, F[hh].z, fmaf(F[hh].x, d0, -F[hh].y)), y[rb][0]);
            y[rb][1] = fmaf(s8, fmaf(-z8, F[hh].z, fmaf(F[hh].x, d8, -F[hh].y)), y[rb][1]);
          }
        }
      }
#pragma unroll
      for (int rb = 0; rb < kRB; ++rb)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          y[rb][i] += __shfl_xor_sync(0xffffffffu, y[rb][i], 1);
          y[rb][i] += __shfl_xor_sync(0xffffffffu, y[rb][i], 2);
        }
      if (t == 0) {
        float* pw = part + ((ph * S + s) * kRowsWarps + warp) * kRU;
#pragma unroll
        for (int rb = 0; rb < kRB; ++rb) {
          pw[16 * rb + g] = y[rb][0];
          pw[16 * rb + g + 8] = y[rb][1];
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(pdone(s));  // release: this warp's partials (and its reads) come first
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
  }
}

// The sum of a K-sliced call: Y[n] = sum over the slices s of ws[s][n] in slice order
// (deterministic), then the bias; launched after the main kernel with programmatic dependent
// launch (griddepcontrol.wait: every slice's partial rows written).
__global__ void __launch_bounds__(256) rows_slice_sum_kernel(const float* __restrict__ ws, int ns, int64_t n_ws,
                                                             int64_t n, const void* bias, tq4_dtype bias_t,
                                                             void* y, tq4_dtype y_t) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int s = 0; s < ns; ++s) v += ws[s * n_ws + i];
    if (bias) v = round_to(v, y_t) + load_as_f32(bias, i, bias_t);
    store_from_f32(y, i, y_t, v);
  }
}

// ---- host side --------------------------------------------------------------------------------

// The scale blocks of a unit's K slice (its 8 packed groups, or the whole row when it has fewer),
// at most the handle's block rows.
static int rows_scale_blocks(const Weight& w) {
  const int64_t nb = (std::min<int64_t>(w.groups, kRowsWarps) * 128 + w.desc.block_size - 1) / w.desc.block_size;
  return (int)std::min<int64_t>(nb, w.blocks_pad);
}

#ifndef TQ4_ROWS_MAX_SLICES
#define TQ4_ROWS_MAX_SLICES 1024  // K slices of 8 groups the kernel takes (rows of up to 8 * this many groups)
#endif

bool rows_eligible(const Weight& w) {
  return w.rw_ok && w.desc.bits == 4 && w.desc.block_size <= 1024 &&
         (w.groups + kRowsWarps - 1) / kRowsWarps <= TQ4_ROWS_MAX_SLICES;
}

int rows_slices(const Weight& w) { return (int)((w.groups + kRowsWarps - 1) / kRowsWarps); }

static int64_t rows_units(const Weight& w) { return (w.desc.N + kRU - 1) / kRU; }

int64_t rows_ws_floats(const Weight& w) {
  return rows_slices(w) > 1 ? rows_slices(w) * rows_units(w) * kRU : 0;
}

int64_t rows_counters(const Weight& w) { return rows_slices(w); }

tq4_status make_rows_maps(Weight& w) {
  w.rw_ok = false;
  // a slice of 8 groups (1024 k) holds whole blocks up to 1024
  if (w.desc.bits != 4 || w.desc.block_size > 1024) return TQ4_OK;
  const int st = dtype_size(w.desc.dequant_dtype);
  const CUtensorMapDataType sdt = st == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const int nbs = rows_scale_blocks(w);
  TQ4_TRY(make_map(&w.rw_wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q.ptr, w.row_bytes, w.n_pad, w.row_bytes, 64, kRU,
                   CU_TENSOR_MAP_SWIZZLE_NONE));
  TQ4_TRY(make_map(&w.rw_smap, sdt, w.scales.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, kSR, nbs,
                   CU_TENSOR_MAP_SWIZZLE_NONE));
  if (w.zps.ptr)
    TQ4_TRY(make_map(&w.rw_zmap, sdt, w.zps.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, kSR, nbs,
                     CU_TENSOR_MAP_SWIZZLE_NONE));
  else
    w.rw_zmap = w.rw_smap;  // never loaded
  w.rw_ok = true;
  return TQ4_OK;
}

struct RowsPlan {
  int stages, stage_bytes, sc_off, zc_off, part_off, tail_off, smem, grid;
};

static RowsPlan plan_rows(const Weight& w) {
  RowsPlan pl{};
  const int st = dtype_size(w.desc.dequant_dtype);
  const int nbs = rows_scale_blocks(w);
  const int sc_bytes = (kSR * nbs * st + 127) / 128 * 128;
  pl.sc_off = (int)std::min<int64_t>(w.groups, kRowsWarps) * kRU * 64;
  pl.zc_off = pl.sc_off + sc_bytes;
  pl.stage_bytes = (pl.zc_off + (w.zps.ptr ? sc_bytes : 0) + 1023) / 1024 * 1024;
  const int per_stage = pl.stage_bytes + 2 * kRowsWarps * kRU * 4;  // + the stage's partials (two laps)
  pl.stages = std::min(kRowsMaxStages, (kRowsSmemBudget - kRowsTail) / per_stage);
  pl.part_off = pl.stages * pl.stage_bytes;
  pl.tail_off = pl.part_off + 2 * pl.stages * kRowsWarps * kRU * 4;
  pl.smem = pl.tail_off + kRowsTail;
  // a multiple of the slice count, each slice's CTAs no more than its units
  const int ns = rows_slices(w);
  const int64_t per_slice = std::min<int64_t>(rows_units(w), std::max(1, kRowsCtas * w.num_sms / ns));
  pl.grid = (int)(per_slice * ns);
  return pl;
}

template <tq4_dtype AT, int SPS>
static cudaError_t launch_rows_t(const Weight& w, const RowsArgs& args, int grid, int smem, cudaStream_t st) {
  auto kern = gemv_rows_kernel<AT, SPS>;
  static std::atomic<uint64_t> attr_set{0};  // per device, once per instantiation
  {
    const cudaError_t e = set_smem_limit_once(kern, kRowsSmemBudget + 1024, attr_set);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(kern, dim3(grid), dim3(kRowsThreads), smem + 1024, st, w.rw_wmap, w.rw_smap, w.rw_zmap, args);
}

template <tq4_dtype AT>
static cudaError_t launch_rows_at(const Weight& w, const RowsArgs& args, int grid, int smem, cudaStream_t st) {
  switch (std::min<int>(w.desc.block_size, 128) / 16) {
    case 1: return launch_rows_t<AT, 1>(w, args, grid, smem, st);
    case 2: return launch_rows_t<AT, 2>(w, args, grid, smem, st);
    case 4: return launch_rows_t<AT, 4>(w, args, grid, smem, st);
    default: return launch_rows_t<AT, 8>(w, args, grid, smem, st);
  }
}

tq4_status run_gemv_rows(const Weight& w, const void* a, tq4_dtype a_t, const void* bias, tq4_dtype bias_t,
                         tq4_dtype y_t, const RowsDst& dst, int* counter, cudaStream_t st, const RowsNorm* norm,
                         float* ws) {
  if (!rows_eligible(w)) {
    set_error("GEMV: the handle has no 32-row unit descriptors");
    return TQ4_ERR_UNSUPPORTED;
  }
  if (dst.ndst < 1 || dst.ndst > kRowsMaxDst || counter == nullptr) {
    set_error("GEMV: bad destinations or no counter");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (norm && a_t != TQ4_F32) {
    set_error("GEMV: the RMSNorm prologue takes f32 activations");
    return TQ4_ERR_UNSUPPORTED;
  }
  const int ns = rows_slices(w);
  if (ns > 1 && (norm || dst.ndst != 1 || dst.epoch || ws == nullptr)) {
    set_error("GEMV: K-sliced rows take one destination, no prologue, and a workspace");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  const RowsPlan pl = plan_rows(w);
  if (pl.stages < 2) {
    set_error("GEMV: a 32-row unit does not fit shared memory");
    return TQ4_ERR_UNSUPPORTED;
  }
  RowsArgs args{};
  args.a = a;
  args.bias = bias;
  args.bias_t = bias_t;
  args.y_t = y_t;
  for (int d = 0; d < dst.ndst; ++d) args.y[d] = dst.y[d];
  args.ndst = dst.ndst;
  args.col0 = dst.col0;
  args.epoch = dst.epoch;
  args.half_elems = dst.half_elems;
  if (norm) {
    args.norm_w = norm->w;
    args.norm_eps = norm->eps;
  }
  args.z_const = w.z_const;
  args.has_zp = w.zps.ptr != nullptr;
  args.st_bytes = dtype_size(w.desc.dequant_dtype);
  args.st_bf16 = w.desc.dequant_dtype == TQ4_BF16;
  args.K = (int)w.desc.K;
  args.N = (int)w.desc.N;
  args.groups = (int)w.groups;
  args.bs_log2 = w.bs_log2;
  args.nbs = rows_scale_blocks(w);
  args.units = (int)((w.desc.N + kRU - 1) / kRU);
  args.stages = pl.stages;
  args.stage_bytes = pl.stage_bytes;
  args.sc_off = pl.sc_off;
  args.zc_off = pl.zc_off;
  args.part_off = pl.part_off;
  args.tail_off = pl.tail_off;
  args.counter = counter;
  args.slices = ns;
  args.ws = ws;
  cudaError_t e;
  switch (a_t) {
    case TQ4_F16: e = launch_rows_at<TQ4_F16>(w, args, pl.grid, pl.smem, st); break;
    case TQ4_BF16: e = launch_rows_at<TQ4_BF16>(w, args, pl.grid, pl.smem, st); break;
    default: e = launch_rows_at<TQ4_F32>(w, args, pl.grid, pl.smem, st); break;
  }
  if (e == cudaSuccess && ns > 1) {
    const int64_t n = w.desc.N;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, 2 * w.num_sms);
    e = launch_pdl(rows_slice_sum_kernel, dim3(grid), dim3(256), 0, st, static_cast<const float*>(ws), ns,
                   rows_units(w) * kRU, n, bias, bias_t, dst.y[0], y_t);
  }
  if (e != cudaSuccess) {
    set_error("GEMV (32-row units) launch failed: %s", cudaGetErrorString(e));
    return TQ4_ERR_CUDA;
  }
  return TQ4_OK;
}

}  // namespace tq4
