// Fused unpack + dequantize + GEMV for decode-shaped MatMulNBits calls (M <= 16).
//
// Math (the MatMulNBits clause, quantized.ex:30-46 with dequantize_weight/4 at :234-240):
//   Y[m][n] = sum_k A[m][k] * (q[n][k] - z[n][b(k)]) * s[n][b(k)]
// is evaluated per "segment" (a run of seg = min(block_size, group, 128) weights of one block).
// The weights enter the tensor cores as magic-number floats O + q/c(k) straight out of one LOP3
// (O = 1024 for f16, 128 for bf16; c(k) is 1/16, 1/4, ... for the nibbles the mask leaves
// shifted, and the staged activation at k is multiplied by c(k) to match). With the staged
// activations v(k) = RN(A[m][k] / E * c(k)) (E an exact power of two per segment chosen so that
// v cannot overflow f16),
//   P[m][n][seg] = sum_{k in seg} (O + q/c(k)) v(k)            (mma.sync, f32 accumulate)
//   Y[m][n]     += s[n][b] * ( E*P - E*O*SV - z[n][b] * E*SA ),  SV = sum v, SA = sum v/c
// so zero points, scales and the magic offset cost a few FMAs per segment and each pair of
// weights costs one LOP3 (plus one shift per 32-bit word).
//
// Structure: persistent CTAs of one TMA producer warp and 8 consumer warps walk "items" (128
// weight rows x a K range). The producer streams each item's packed rows (one 128-row x 64-byte
// box per group, so consumer reads of rows 64 bytes apart are bank-conflict free) and the
// block-major scales / zero points of the same K range into a ring of mbarrier stages; it runs
// ahead into the next item while the consumers finish the current one. Each consumer warp owns 16
// rows (mma.sync m16n8k16, weights as the A operand). Activations are staged in shared memory once
// per K range.
//   M = 1: the MMA's 8 activation columns hold 8 different segments of the one activation row
//          (column c takes segment c of the stage, the others see zero), so scales and zero points
//          are applied once per stage (up to 8 segments) instead of once per segment.
//   M > 1: the columns are activation rows; the correction runs at the end of each segment.
// Items that share rows (split-K) reduce through a float workspace: the last CTA of a row tile
// sums the partials in a fixed order (deterministic) and resets its counter.
#include <map>
#include <memory>
#include <mutex>

#include "fragments.cuh"
#include "internal.cuh"
#include "rows.cuh"
#include "sm100.cuh"

namespace tq4 {

constexpr int kRows = 128;            // weight rows per item (8 consumer warps x 16)
constexpr int kScaleRows = 136;       // scale box height: 128 rows + 8 of padding (bank spread)
constexpr int kConsumers = 256;
constexpr int kGemvThreads = kConsumers + 32;
constexpr int kMaxStages = 4;
constexpr int kSmemBudget = 110 * 1024;  // two CTAs per SM

enum GemvMode { kCols = 0, kSegMT1 = 1, kSegMT2 = 2 };

struct GemvArgs {
  const void* a;
  const void* bias;
  tq4_dtype bias_t;
  void* y;
  tq4_dtype y_t;
  int64_t ldy;
  float z_const;
  int has_zp;
  int st_bytes, st_bf16;
  int K, N, M;
  int bs_log2, seg_log2;
  int groups;            // groups per row
  int groups_per_split;  // item K range in groups
  int gps;               // groups per stage
  int nbs;               // scale blocks per stage (box height)
  int stages;
  int stage_bytes, sc_off, zc_off;  // within a stage
  int act_off, seg_off, bar_off;    // within the CTA's shared memory
  int sk;                // staged activation row stride (elements)
  int ctas_n;            // row tiles of 128
  int ksplit;
  int items;
  int units;             // M = 1 stream-K: (row tile, stage) units, stages per row tile, max pieces
  int spr;
  int maxp;
  int dyn;               // M = 1: whole row tiles handed out by an arrival counter (no partials)
  int pre, bf_off;       // M = 1: B fragments prebuilt per CTA at bf_off (0: masked in the loop)
  int clu, gpc;          // M = 1: a row tile's K split over a cluster of `clu` CTAs, gpc groups each
  // M = 1, f32 activations: a transform applied while staging (decoder fusion). 1: RMSNorm,
  // a = x * rsqrt(mean(x^2) + eps) * pro_w; 2: SwiGLU, a = silu(x) * pro_b (K values each).
  int pro;
  const float* pro_w;
  const float* pro_b;
  float pro_eps;
  int64_t n_pad;
  float* ws;
  int* counters;
};

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

// Stages A[0:M][k0 : k0+kr] into shared memory as v(k) = RN(A / E * c(k)) in the MMA type, with
// the per-segment factors {E, E*O*SV + (no zero points ? z*E*SA : 0), E*SA} as float4 [seg][mp].
// Rows >= M are left as they are: their outputs are never stored, and an MMA output element
// depends only on its own activation row. Run by the 256 consumer threads. `act` and `segf`
// point at position k0 (element k0 - kk is at act[kk]). PRECISE must match the weight_pairs
// variant the consumers use.
//
// With BF_SPS > 0 (M = 1, the whole row, k0 = 0) each 4-value run also lands in the prebuilt B
// fragment table `bfw` (uint2 units, zero-filled beforehand): 16-k slice ks, lane
// 4 * ((ks / BF_SPS) % BF_NSEG) + (k / 4) % 4, half ks % 2 of slice pair ks / 2.
template <int BITS, tq4_dtype AT, bool PRECISE = (AT == TQ4_F32), int BF_SPS = 0, int BF_NSEG = 8>
__device__ __forceinline__ void stage_activations(const GemvArgs& p, int k0, int kr, int mp,
                                                  uint16_t* act, float4* segf, float pro_rs = 1.f,
                                                  uint2* bfw = nullptr) {
  constexpr bool BF = (AT == TQ4_BF16);
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int vec_per_row = kr / 4;
  const int total = p.M * vec_per_row;
  const int total_pad = (total + 31) & ~31;  // whole warps take part in the shuffles
  const int L = (1 << p.seg_log2) >> 2;      // lanes per segment (<= 32)
  const bool vec = (p.K & 3) == 0;
  const float O = magic_offset<BITS, BF, PRECISE>();
  const bool fold_z = !p.has_zp;
  for (int base = 0; base < total_pad; base += 4 * kConsumers) {
    float a4[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {  // issue all loads first
      const int v = base + u * kConsumers + tid;
      if (v < total) {
        const int64_t k = (int64_t)k0 + (v % vec_per_row) * 4;
        load_act4<AT>(p.a, v / vec_per_row, k, p.K, vec, a4[u]);
        if constexpr (AT == TQ4_F32) {
          if (p.pro == 1) {  // RMSNorm (the row's factor computed by the caller)
#pragma unroll
            for (int e = 0; e < 4; ++e) a4[u][e] = (k + e < p.K) ? a4[u][e] * pro_rs * p.pro_w[k + e] : 0.f;
          } else if (p.pro == 2) {  // SwiGLU
            float b4[4];
            load_act4<TQ4_F32>(p.pro_b, 0, k, p.K, vec, b4);
#pragma unroll
            for (int e = 0; e < 4; ++e) a4[u][e] = a4[u][e] / (1.f + expf(-a4[u][e])) * b4[e];
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) a4[u][e] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (base + u * kConsumers + warp * 32 >= total_pad) continue;  // warp-uniform
      const int v = base + u * kConsumers + tid;
      const int m = v / vec_per_row, kk = (v % vec_per_row) * 4;
      float mx = fmaxf(fmaxf(fabsf(a4[u][0]), fabsf(a4[u][1])), fmaxf(fabsf(a4[u][2]), fabsf(a4[u][3])));
      for (int off = 1; off < L; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      float e_scale = 1.f, inv = 1.f;
      if (mx > 0.f && mx <= 3.402823466e38f) {
        // mx = f * 2^ex with f in [0.5, 1): ex = biased exponent - 126 (subnormals clamp below)
        const int ex = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 126;
        const int s = max(-126, min(127, ex - 15));  // mx / 2^s in [2^14, 2^15)
        e_scale = __uint_as_float((uint32_t)(s + 127) << 23);
        inv = s < 127 ? __uint_as_float((uint32_t)(127 - s) << 23) : 5.8774717541e-39f;  // 2^-s
      }
      uint16_t h[4];
      float sv = 0.f, sa = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float c = act_factor<BITS, BF, PRECISE>(kk + e);  // kk: a multiple of 4
        const float c_inv = act_factor_inv<BITS, BF, PRECISE>(kk + e);
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
        sa += val * c_inv;  // exact: c is a power of two
      }
      for (int off = 1; off < L; off <<= 1) {
        sv += __shfl_xor_sync(0xffffffffu, sv, off);
        sa += __shfl_xor_sync(0xffffffffu, sa, off);
      }
      if (v < total) {
        uint2 packed;
        packed.x = (uint32_t)h[0] | ((uint32_t)h[1] << 16);
        packed.y = (uint32_t)h[2] | ((uint32_t)h[3] << 16);
        *reinterpret_cast<uint2*>(act + m * p.sk + kk) = packed;
        if constexpr (BF_SPS > 0) {
          const int ks = kk >> 4;
          const int dst = ((ks >> 1) * 32 + 4 * ((ks / BF_SPS) % BF_NSEG) + ((kk >> 2) & 3)) * 2 + (ks & 1);
          bfw[dst] = packed;
        }
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

// The item's K range.
struct ItemRange {
  int rt, split, g_begin, g_end, k0, kr;
};
__device__ __forceinline__ ItemRange item_range(const GemvArgs& p, int item, int G) {
  ItemRange r;
  r.split = item / p.ctas_n;
  r.rt = item % p.ctas_n;
  r.g_begin = r.split * p.groups_per_split;
  r.g_end = min(p.groups, r.g_begin + p.groups_per_split);
  r.k0 = r.g_begin * G;
  r.kr = (r.g_end - r.g_begin) * G;
  return r;
}

// sum_{i < n} src[i * stride] in index order, with the loads issued 16 at a time.
__device__ __forceinline__ float sum_partials(const float* src, int64_t stride, int n) {
  float total = 0.f;
  for (int base = 0; base < n; base += 16) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = (base + i < n) ? __ldcg(src + (base + i) * stride) : 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) total += v[i];
  }
  return total;
}

// Y (or a split-K partial) of one output.
__device__ __forceinline__ void write_out(const GemvArgs& p, int split, int64_t n, int m, float v) {
  if (p.ksplit == 1) {
    if (n < p.N && m < p.M) {
      if (p.bias) v = round_to(v, p.y_t) + load_as_f32(p.bias, n, p.bias_t);
      store_from_f32(p.y, (int64_t)m * p.ldy + n, p.y_t, v);
    }
  } else if (m < p.M) {
    p.ws[((int64_t)split * p.M + m) * p.n_pad + n] = v;
  }
}

template <int BITS, tq4_dtype AT, int MODE>
__global__ void __launch_bounds__(kGemvThreads, 2)
    gemv_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_s,
                const __grid_constant__ CUtensorMap map_z, const GemvArgs p) {
  constexpr bool BF = (AT == TQ4_BF16);
  constexpr bool PRECISE = (AT == TQ4_F32);
  constexpr int G = 512 / BITS;  // elements per 64-byte group
  constexpr int STEPS = G / 16;
  constexpr int STEPS_PER_WORD = 32 / BITS / 4;  // 2 (4-bit), 4 (2-bit), 1 (8-bit)
  constexpr int MT = (MODE == kSegMT2) ? 2 : 1;
  constexpr int MP = (MODE == kCols) ? 1 : 8 * MT;  // staged activation rows
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_last;
  // stages start 1024-byte aligned (TMA destinations)
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t sbase = (raw_addr + 1023) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw_addr);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t bars = sbase + p.bar_off;
  const int S = p.stages;
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (kMaxStages + s); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.bar_off + 8 * 2 * kMaxStages);

  // this CTA's items: a contiguous range, so consecutive items mostly share their K range
  const int it0 = (int)((int64_t)blockIdx.x * p.items / gridDim.x);
  const int it1 = (int)((int64_t)(blockIdx.x + 1) * p.items / gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 8);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int gs = 0;  // global stage counter (same sequence as the consumers)
      bool ok = true;
      for (int item = it0; item < it1 && ok; ++item) {
        const ItemRange r = item_range(p, item, G);
        const int row0 = r.rt * kRows;
        for (int c0 = r.g_begin; c0 < r.g_end; c0 += p.gps, ++gs) {
          const int s = gs % S;
          if (!mbar_wait(empty(s), ((gs / S) & 1) ^ 1, abort_flag, kDevTimeoutStageEmpty)) {
            ok = false;
            break;
          }
          const int ng = min(p.gps, r.g_end - c0);
          const int b0 = (c0 * G) >> p.bs_log2;
          const uint32_t st = sbase + s * p.stage_bytes;
          const uint32_t sc_bytes = kScaleRows * p.nbs * p.st_bytes;
          mbar_expect_tx(full(s), ng * kRows * 64 + sc_bytes * (p.has_zp ? 2 : 1));
          for (int gi = 0; gi < ng; ++gi) tma_load_2d(st + gi * kRows * 64, &map_w, (c0 + gi) * 64, row0, full(s));
          tma_load_2d(st + p.sc_off, &map_s, row0, b0, full(s));
          if (p.has_zp) tma_load_2d(st + p.zc_off, &map_z, row0, b0, full(s));
        }
      }
      // the copies still in flight land before the CTA exits (bounded)
      for (int g = max(0, gs - S); g < gs; ++g) mbar_drain(full(g % S), (g / S) & 1);
    }
    return;  // the producer takes part in no consumer barrier
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const int rl = warp * 16 + g;  // this thread's first row within the item
  uint16_t* act = reinterpret_cast<uint16_t*>(smem + p.act_off);
  float4* segf = reinterpret_cast<float4*>(smem + p.seg_off);
  const int seg_log2 = p.seg_log2;
  const int seg = 1 << seg_log2;
  int gs = 0;
  int staged_split = -1;
  bool ok = true;

  for (int item = it0; item < it1; ++item) {
    const ItemRange r = item_range(p, item, G);
    if (r.split != staged_split) {  // activations for this K range
      consumer_sync();              // everyone is done with the previous range
      stage_activations<BITS, AT>(p, r.k0, r.kr, MP, act, segf);
      staged_split = r.split;
      consumer_sync();
    }

    float acc[MT][4];   // kSeg*: finished outputs; kCols: per-thread partial sums of 2 rows
    float blk[MT][4];   // MMA accumulators
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][i] = blk[mt][i] = 0.f;

    for (int c0 = r.g_begin; c0 < r.g_end; c0 += p.gps, ++gs) {
      const int s = gs % S;
      if (ok) ok = mbar_wait(full(s), (gs / S) & 1, abort_flag, kDevTimeoutTmaFull);
      if (ok) {
        const int ng = min(p.gps, r.g_end - c0);
        const uint8_t* st = smem + s * p.stage_bytes;
        const uint8_t* sc = st + p.sc_off;
        const uint8_t* zc = st + p.zc_off;
        const int b0 = (c0 * G) >> p.bs_log2;
        const int ks = (c0 - r.g_begin) * G;  // stage start within the staged activations
        for (int gi = 0; gi < ng; ++gi) {
          const uint4 xa = *reinterpret_cast<const uint4*>(st + gi * kRows * 64 + rl * 64 + t * 16);
          const uint4 xb = *reinterpret_cast<const uint4*>(st + gi * kRows * 64 + (rl + 8) * 64 + t * 16);
#pragma unroll
          for (int j = 0; j < STEPS; ++j) {
            const int w = j / STEPS_PER_WORD;
            uint32_t a0, a1, a2, a3;
            weight_pairs<BITS, BF, PRECISE>(word_of(xa, w), j, a0, a2);
            weight_pairs<BITS, BF, PRECISE>(word_of(xb, w), j, a1, a3);
            const int kk = ks + gi * G + 16 * j + 4 * t;
            if constexpr (MODE == kCols) {
              // column g takes segment g of the stage; the other columns see zero
              const int col = (gi * G + 16 * j) >> seg_log2;
              const uint2 bv = *reinterpret_cast<const uint2*>(act + kk);
              const bool mine = (g == col);
              mma16816<BF>(blk[0], a0, a1, a2, a3, mine ? bv.x : 0u, mine ? bv.y : 0u);
            } else {
#pragma unroll
              for (int mt = 0; mt < MT; ++mt) {
                const uint2 bv = *reinterpret_cast<const uint2*>(act + (mt * 8 + g) * p.sk + kk);
                mma16816<BF>(blk[mt], a0, a1, a2, a3, bv.x, bv.y);
              }
              if ((((j + 1) * 16) & (seg - 1)) == 0) {  // end of a segment
                const int kseg = ks + gi * G + (j + 1) * 16 - seg;  // within the staged range
                const int s_idx = kseg >> seg_log2;
                const int lb = ((r.k0 + kseg) >> p.bs_log2) - b0;
                const float s_g = scale_to_f32(sc, lb * kScaleRows + rl, p.st_bytes, p.st_bf16);
                const float s_g8 = scale_to_f32(sc, lb * kScaleRows + rl + 8, p.st_bytes, p.st_bf16);
                const float z_g = p.has_zp ? scale_to_f32(zc, lb * kScaleRows + rl, p.st_bytes, p.st_bf16) : 0.f;
                const float z_g8 = p.has_zp ? scale_to_f32(zc, lb * kScaleRows + rl + 8, p.st_bytes, p.st_bf16) : 0.f;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                  const int m0 = mt * 8 + 2 * t;
                  const float4 F0 = segf[s_idx * MP + m0], F1 = segf[s_idx * MP + m0 + 1];
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
        }
        if constexpr (MODE == kCols) {
          // columns 2t and 2t+1 hold segments 2t and 2t+1 of this stage
          const int nseg_stage = (ng * G) >> seg_log2;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int sg = 2 * t + h;
            if (sg < nseg_stage) {
              const int kseg = ks + (sg << seg_log2);
              const int lb = ((r.k0 + kseg) >> p.bs_log2) - b0;
              const float4 F = segf[kseg >> seg_log2];
              const float s_g = scale_to_f32(sc, lb * kScaleRows + rl, p.st_bytes, p.st_bf16);
              const float s_g8 = scale_to_f32(sc, lb * kScaleRows + rl + 8, p.st_bytes, p.st_bf16);
              float z_g = 0.f, z_g8 = 0.f;
              if (p.has_zp) {
                z_g = scale_to_f32(zc, lb * kScaleRows + rl, p.st_bytes, p.st_bf16);
                z_g8 = scale_to_f32(zc, lb * kScaleRows + rl + 8, p.st_bytes, p.st_bf16);
              }
              acc[0][0] = fmaf(s_g, fmaf(-z_g, F.z, fmaf(F.x, blk[0][h], -F.y)), acc[0][0]);
              acc[0][2] = fmaf(s_g8, fmaf(-z_g8, F.z, fmaf(F.x, blk[0][2 + h], -F.y)), acc[0][2]);
            }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) blk[0][i] = 0.f;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(s));  // this warp is done with the stage
    }

    // ---- outputs of the item: rows row0 + rl (and + 8)
    const int64_t n_g = (int64_t)r.rt * kRows + rl, n_g8 = n_g + 8;
    if constexpr (MODE == kCols) {
      float y0 = acc[0][0], y8 = acc[0][2];
      y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
      y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
      y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
      y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
      if (t == 0) {
        write_out(p, r.split, n_g, 0, y0);
        write_out(p, r.split, n_g8, 0, y8);
      }
    } else {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          write_out(p, r.split, (i < 2) ? n_g : n_g8, mt * 8 + 2 * t + (i & 1), acc[mt][i]);
    }
    if (p.ksplit > 1) {
      // the last item of a row tile sums the partials in split order
      __threadfence();
      consumer_sync();
      if (threadIdx.x == 0) {
        const int prev = atomicAdd(&p.counters[r.rt], 1);
        s_last = (prev == p.ksplit - 1);
        if (prev >= p.ksplit) report(kDevTimeoutSplitK);  // a counter left non-zero earlier
      }
      consumer_sync();
      if (s_last) {
        __threadfence();
        for (int i = threadIdx.x; i < kRows * p.M; i += kConsumers) {
          const int m = i / kRows;
          const int64_t n = (int64_t)r.rt * kRows + (i % kRows);
          if (n >= p.N) continue;
          float v = sum_partials(p.ws + (int64_t)m * p.n_pad + n, (int64_t)p.M * p.n_pad, p.ksplit);
          if (p.bias) v = round_to(v, p.y_t) + load_as_f32(p.bias, n, p.bias_t);
          store_from_f32(p.y, (int64_t)m * p.ldy + n, p.y_t, v);
        }
        if (threadIdx.x == 0) p.counters[r.rt] = 0;
      }
      consumer_sync();
    }
  }
}

// ---- M = 1, 4-bit: compile-time segment layout, stream-K balance -----------------------------------
// SPS = MMA steps (16 weights each) per segment = seg / 16. A stage holds GPS = min(4, SPS) groups
// of 128 weights, i.e. NSEG = GPS * 8 / SPS <= 8 segments; MMA column c takes segment c of the
// stage. Every step's column is a compile-time constant, so a thread's B fragment is the staged
// activation times a 0/1 f16x2 mask (one FMA-pipe multiply) and the block of each segment is its
// index (block_size <= 128, so blocks start on group boundaries). The (row tile, group) units are
// split evenly over the CTAs (stream-K): each CTA stages the whole activation row once and walks
// its units in stages of up to GPS groups that never cross a row tile; a row tile that spans
// several CTAs is finished by the last of them, which sums the partials in CTA order.
__device__ __forceinline__ int unit_owner(int u, int units, int grid) {
  return (int)((((int64_t)u + 1) * grid - 1) / units);
}
__device__ __forceinline__ int unit_first(int b, int units, int grid) {
  return (int)((int64_t)b * units / grid);
}

// HOLD (the stream-K mode): the producer issues one stage, then waits for the activations.
template <tq4_dtype AT, int SPS, bool HOLD>
__global__ void __launch_bounds__(kGemvThreads, 3)
    gemv_m1_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_s,
                   const __grid_constant__ CUtensorMap map_z, const GemvArgs p) {
  constexpr bool BF = (AT == TQ4_BF16);
  // A column accumulates one segment between corrections, so the 1024 offset of the plain magic
  // numbers only costs precision on long segments: f32 activations take the precise weights from
  // 64-wide segments up.
  constexpr bool PRECISE = (AT == TQ4_F32) && SPS > 2;
  constexpr int G = 128;
  constexpr int GPS = SPS < 4 ? SPS : 4;
  constexpr int SEG = 16 * SPS;
  constexpr int NSEG = GPS * 8 / SPS;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_lastv[2];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t sbase = (raw_addr + 1023) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw_addr);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t bars = sbase + p.bar_off;
  const int S = p.stages;
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (kMaxStages + s); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.bar_off + 8 * 2 * kMaxStages);
  volatile int* sinfo = reinterpret_cast<volatile int*>(smem + p.bar_off + 8 * 2 * kMaxStages + 16);  // dyn
  const uint32_t staged = bars + 8 * 2 * kMaxStages + 16 + 8 * kMaxStages;
  int u0, u1;
  if (p.dyn) {
    u0 = 0;
    u1 = p.units;
  } else if (p.clu) {  // row tile blockIdx.x / clu, K share blockIdx.x % clu (its cluster rank)
    const int rt = blockIdx.x / p.clu, kc = blockIdx.x % p.clu;
    u0 = rt * p.groups + min(p.groups, kc * p.gpc);
    u1 = rt * p.groups + min(p.groups, (kc + 1) * p.gpc);
  } else {
    u0 = unit_first(blockIdx.x, p.units, gridDim.x);
    u1 = unit_first(blockIdx.x + 1, p.units, gridDim.x);
  }

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 8);
    }
    if constexpr (HOLD) mbar_init(staged, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    // The packed weights, scales and zero points are constant: the ring starts filling before the
    // previous kernel on the stream has finished (programmatic dependent launch).
    if (lane == 0) {
      const uint32_t sc_bytes = kScaleRows * p.nbs * p.st_bytes;
      int gs = 0;
      auto issue = [&](int s, int rt, int c0, int ng) {
        const int row0 = rt * kRows;
        const uint32_t st = sbase + s * p.stage_bytes;
        mbar_expect_tx(full(s), ng * kRows * 64 + sc_bytes * (p.has_zp ? 2 : 1));
        for (int gi = 0; gi < ng; ++gi) tma_load_2d(st + gi * kRows * 64, &map_w, (c0 + gi) * 64, row0, full(s));
        const int b0 = (c0 * G) >> p.bs_log2;
        tma_load_2d(st + p.sc_off, &map_s, row0, b0, full(s));
        if (p.has_zp) tma_load_2d(st + p.zc_off, &map_z, row0, b0, full(s));
      };
      int s = 0;
      uint32_t ph = 0;  // the ring's current lap parity
      auto advance = [&]() {
        ++gs;
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      };
      if (p.dyn) {
        // Row tile blockIdx.x first (prefetched before the previous kernel finishes), then the
        // tiles gridDim.x, gridDim.x + 1, ... in ticket order: CTAs that stream faster take more.
        // A stage's tag is its (row tile, first group); row tile -1 says there is no more work.
        // Every CTA takes tickets until one fails, so a call takes exactly ctas_n tickets
        // (ctas_n - gridDim.x tiles, gridDim.x failures): the taker of ticket ctas_n - 1 is the
        // call's last and puts the counter back to zero for the next call on the stream. The
        // next ticket is taken when a tile's first stage is issued, off the issue path.
        auto take = [&]() {
          const int v = atomicAdd(&p.counters[0], 1);
          if (v == p.ctas_n - 1) p.counters[0] = 0;
          return (int)gridDim.x + v;
        };
        int rt = blockIdx.x, next = 0;
        bool waited = false, ok = true;
        while (ok) {
          if (rt >= p.ctas_n) {  // no work left: a stage that only says so
            if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, kDevTimeoutStageEmpty)) break;
            sinfo[2 * s] = -1;
            mbar_arrive(full(s));
            advance();
            break;
          }
          for (int c0 = 0; c0 < p.groups && ok; c0 += GPS) {
            ok = mbar_wait(empty(s), ph ^ 1u, abort_flag, kDevTimeoutStageEmpty);
            if (!ok) break;
            sinfo[2 * s] = rt;
            sinfo[2 * s + 1] = c0;
            issue(s, rt, c0, min(GPS, p.groups - c0));
            advance();
            if (c0 == 0 && waited) next = take();
          }
          if (!waited) {
            pdl_wait();  // the counter belongs to the stream's order
            waited = true;
            next = take();
          }
          rt = next;
        }
      } else {
        // Stream-K shares: only the first stage is issued before the activations are staged. A
        // share is a few stages more than the ring holds, and with the ring full the consumers'
        // loads of the activation row queued behind the whole grid's weight copies (clock stamps:
        // 3.5 us to stage 8 KB). Cluster shares fit their rings and are all issued at once.
        int rt = u0 / p.groups, c0 = u0 - rt * p.groups;
        bool held = HOLD;
        for (int u = u0; u < u1;) {
          if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, kDevTimeoutStageEmpty)) break;
          const int ng = min(min(GPS, p.groups - c0), u1 - u);  // a chunk never crosses a row tile
          issue(s, rt, c0, ng);
          advance();
          if (HOLD && held) {
            held = false;
            if (!mbar_wait(staged, 0, abort_flag, kDevTimeoutStaged)) break;
          }
          u += ng;
          c0 += ng;
          if (c0 == p.groups) {
            c0 = 0;
            ++rt;
          }
        }
      }
      for (int g = max(0, gs - S); g < gs; ++g) mbar_drain(full(g % S), (g / S) & 1);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const int rl = warp * 16 + g;
  uint16_t* act = reinterpret_cast<uint16_t*>(smem + p.act_off);
  float4* segf = reinterpret_cast<float4*>(smem + p.seg_off);
  uint4* bf = reinterpret_cast<uint4*>(smem + p.bf_off);
  if (p.pre) {  // the prebuilt fragment table starts as zeros (before the wait: shared memory only)
    for (int i = threadIdx.x; i < p.groups * 128; i += kConsumers) bf[i] = make_uint4(0u, 0u, 0u, 0u);
    consumer_sync();  // before other threads' staging writes land in the same entries
  }
  pdl_wait();  // activations, outputs and partials belong to the stream's order from here on
  float pro_rs = 1.f;
  if (AT == TQ4_F32 && p.pro == 1) {  // RMSNorm prologue: the whole row's mean square
    __shared__ float red[kConsumers / 32];
    const float* x = static_cast<const float*>(p.a);
    float ss = 0.f;
    for (int k = threadIdx.x; k < p.K; k += kConsumers) ss = fmaf(x[k], x[k], ss);
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[warp] = ss;
    consumer_sync();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kConsumers / 32; ++i) tot += red[i];
    pro_rs = 1.f / sqrtf(tot / (float)p.K + p.pro_eps);
  }
  if (u1 > u0) {
    // the activations of the groups this CTA's units touch (one or two runs, or the whole row)
    const int c_a = u0 % p.groups, c_b = (u1 - 1) % p.groups;
    if (p.pre) {
      stage_activations<4, AT, PRECISE, SPS, NSEG>(p, 0, p.groups * G, 1, act, segf, pro_rs,
                                                   reinterpret_cast<uint2*>(bf));
    } else if (u1 - u0 >= p.groups) {
      stage_activations<4, AT, PRECISE>(p, 0, p.groups * G, 1, act, segf, pro_rs);
    } else if (c_a <= c_b) {
      stage_activations<4, AT, PRECISE>(p, c_a * G, (c_b - c_a + 1) * G, 1, act + c_a * G,
                                        segf + (c_a * G) / SEG, pro_rs);
    } else {
      stage_activations<4, AT, PRECISE>(p, c_a * G, (p.groups - c_a) * G, 1, act + c_a * G,
                                        segf + (c_a * G) / SEG, pro_rs);
      stage_activations<4, AT, PRECISE>(p, 0, (c_b + 1) * G, 1, act, segf, pro_rs);
    }
  }
  consumer_sync();
  if constexpr (HOLD) {
    if (threadIdx.x == 0) mbar_arrive(staged);
  }

  // Prebuilt B fragments (the lm_head's row-tile hand-out, where a CTA reuses them for every
  // row tile it takes): MMA column c takes the segments s with s % NSEG == c (an absolute
  // assignment), and a lane's B fragment of 16-k slice ks is its four staged activations when
  // its column g is the slice's, else zero: the 0/1 column mask applied once per CTA instead of
  // in every MMA step. Layout [group][slice pair][lane] of uint4 (slices 2i, 2i+1): one 16-byte
  // load per two MMAs.
  const uint4* bfq = bf + lane;

  // 0/1 multipliers of this thread's B column for each stage column (stages relative)
  const uint32_t one2 = BF ? 0x3F803F80u : 0x3C003C00u;
  uint32_t mask[NSEG];
#pragma unroll
  for (int c = 0; c < NSEG; ++c) mask[c] = (g == c) ? one2 : 0u;

  int s = 0;
  uint32_t ph = 0;  // the ring's current lap parity
  bool ok = true;
  float acc0 = 0.f, acc8 = 0.f;
  int npub = 0, pub_rt[2] = {0, 0}, pub_pieces[2] = {0, 0};
  int rt = u0 / p.groups, c0 = u0 - rt * p.groups, ng = 0;  // walk of the static modes
  for (int u = u0; u < u1;) {
    if (p.dyn) {
      if (!mbar_wait(full(s), ph, abort_flag, kDevTimeoutTmaFull)) break;
      rt = sinfo[2 * s];
      if (rt < 0) break;  // the producer ran out of row tiles
      c0 = sinfo[2 * s + 1];
      ng = min(GPS, p.groups - c0);
    } else {
      if (ng > 0) {  // the previous stage's groups
        c0 += ng;
        if (c0 == p.groups) {
          c0 = 0;
          ++rt;
        }
      }
      ng = min(min(GPS, p.groups - c0), u1 - u);
      u += ng;
      if (ok) ok = mbar_wait(full(s), ph, abort_flag, kDevTimeoutTmaFull);
    }
    if (ok) {
      const uint8_t* st = smem + s * p.stage_bytes;
      const uint8_t* sc = st + p.sc_off;
      const uint8_t* zc = st + p.zc_off;
      const uint16_t* actk = act + c0 * G + 4 * t;
      const uint4* bq = bfq + c0 * 128;
      float blk2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // even / odd steps
      if (p.pre) {
#pragma unroll
        for (int gi = 0; gi < GPS; ++gi) {
          if (gi < ng) {
            const uint4 xa = *reinterpret_cast<const uint4*>(st + gi * kRows * 64 + rl * 64 + t * 16);
            const uint4 xb = *reinterpret_cast<const uint4*>(st + gi * kRows * 64 + (rl + 8) * 64 + t * 16);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const uint4 bb = bq[(gi * 4 + j / 2) * 32];
              uint32_t a0, a1, a2, a3;
              weight_pairs<4, BF, PRECISE>(word_of(xa, j / 2), j, a0, a2);
              weight_pairs<4, BF, PRECISE>(word_of(xb, j / 2), j, a1, a3);
              mma16816<BF>(blk2[0], a0, a1, a2, a3, bb.x, bb.y);
              weight_pairs<4, BF, PRECISE>(word_of(xa, j / 2), j + 1, a0, a2);
              weight_pairs<4, BF, PRECISE>(word_of(xb, j / 2), j + 1, a1, a3);
              mma16816<BF>(blk2[1], a0, a1, a2, a3, bb.z, bb.w);
            }
          }
        }
      } else {
#pragma unroll
      for (int gi = 0; gi < GPS; ++gi) {
        if (gi < ng) {
          const uint4 xa = *reinterpret_cast<const uint4*>(st + gi * kRows * 64 + rl * 64 + t * 16);
          const uint4 xb = *reinterpret_cast<const uint4*>(st + gi * kRows * 64 + (rl + 8) * 64 + t * 16);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint32_t a0, a1, a2, a3;
            weight_pairs<4, BF, PRECISE>(word_of(xa, j / 2), j, a0, a2);
            weight_pairs<4, BF, PRECISE>(word_of(xb, j / 2), j, a1, a3);
            const uint2 bv = *reinterpret_cast<const uint2*>(actk + gi * G + 16 * j);
            const uint32_t m = mask[(gi * 8 + j) / SPS];
            uint32_t b0, b1;
            if (BF) {
              asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(b0) : "r"(bv.x), "r"(m));
              asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(b1) : "r"(bv.y), "r"(m));
            } else {
              asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(b0) : "r"(bv.x), "r"(m));
              asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(b1) : "r"(bv.y), "r"(m));
            }
            mma16816<BF>(blk2[j & 1], a0, a1, a2, a3, b0, b1);  // two independent MMA chains
          }
        }
      }
      }
      float blk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) blk[i] = blk2[0][i] + blk2[1][i];
      // Column c = 2t + h holds the stage's segment (c - s0) mod NSEG: s0 is the stage's first
      // segment with prebuilt fragments (absolute columns), 0 when masked in the loop.
      const int nseg = ng * 8 / SPS;
      const int s0 = p.pre ? (c0 * (8 / SPS)) % NSEG : 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int sg = (2 * t + h - s0 + NSEG) % NSEG;
        if (2 * t + h < NSEG && sg < nseg) {
          const int lb = (sg * SEG) >> p.bs_log2;  // the stage starts on a block boundary
          const float4 F = segf[(c0 * G) / SEG + sg];
          const float s_g = scale_to_f32(sc, lb * kScaleRows + rl, p.st_bytes, p.st_bf16);
          const float s_g8 = scale_to_f32(sc, lb * kScaleRows + rl + 8, p.st_bytes, p.st_bf16);
          float z_g = 0.f, z_g8 = 0.f;
          if (p.has_zp) {
            z_g = scale_to_f32(zc, lb * kScaleRows + rl, p.st_bytes, p.st_bf16);
            z_g8 = scale_to_f32(zc, lb * kScaleRows + rl + 8, p.st_bytes, p.st_bf16);
          }
          acc0 = fmaf(s_g, fmaf(-z_g, F.z, fmaf(F.x, blk[h], -F.y)), acc0);
          acc8 = fmaf(s_g8, fmaf(-z_g8, F.z, fmaf(F.x, blk[2 + h], -F.y)), acc8);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty(s));
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }

    // end of this CTA's piece of row tile rt
    if (!p.clu && (c0 + ng == p.groups || u == u1)) {
      float y0 = acc0, y8 = acc8;
      y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
      y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
      y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
      y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
      acc0 = acc8 = 0.f;
      const int64_t n_g = (int64_t)rt * kRows + rl;
      const int b_first = p.dyn ? 0 : unit_owner(rt * p.groups, p.units, gridDim.x);
      const int b_last = p.dyn ? 0 : unit_owner(rt * p.groups + p.groups - 1, p.units, gridDim.x);
      if (b_first == b_last) {  // the whole row tile is this CTA's
        if (t == 0) {
          write_out(p, 0, n_g, 0, y0);
          write_out(p, 0, n_g + 8, 0, y8);
        }
      } else if (npub < 2) {  // only the first and the last piece of a CTA can be shared
        const int piece = blockIdx.x - b_first;
        float* part = p.ws + ((int64_t)rt * p.maxp + piece) * kRows;
        if (t == 0) {
          part[rl] = y0;
          part[rl + 8] = y8;
        }
        pub_rt[npub] = rt;  // published after the loop: one fence, off the weight stream
        pub_pieces[npub] = b_last - b_first + 1;
        ++npub;
      }
    }
  }

  if (p.clu) {
    // The cluster's partials of row tile blockIdx.x / clu: each CTA leaves its 128 sums in its
    // shared memory; the rank-0 CTA adds them in rank order (deterministic) and writes Y; the
    // second barrier keeps every CTA's shared memory alive until then.
    __shared__ float red_s[kRows];
    float y0 = acc0, y8 = acc8;
    y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
    y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
    y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
    y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
    if (t == 0) {
      red_s[rl] = y0;
      red_s[rl + 8] = y8;
    }
    cluster_sync_all();
    if (cluster_ctarank() == 0 && threadIdx.x < kRows) {
      float v = 0.f;
      for (int r = 0; r < p.clu; ++r) v += ld_cluster_f32(red_s + threadIdx.x, (unsigned)r);
      const int64_t n = (int64_t)(blockIdx.x / p.clu) * kRows + threadIdx.x;
      if (n < p.N) {
        if (p.bias) v = round_to(v, p.y_t) + load_as_f32(p.bias, n, p.bias_t);
        store_from_f32(p.y, n, p.y_t, v);
      }
    }
    cluster_sync_all();
    return;
  }

  if (p.dyn) return;  // the producer's last ticket put the counter back

  // Publish the shared pieces: after a consumer barrier one thread fences (making every
  // consumer's partial stores visible) and counts the arrivals; the last CTA of a row tile sums
  // its partials in CTA order and resets the counter.
  if (npub > 0) {
    consumer_sync();
    if (threadIdx.x == 0) {
      __threadfence();
      bool any = false;
      for (int i = 0; i < npub; ++i) {
        const int prev = atomicAdd(&p.counters[pub_rt[i]], 1);
        s_lastv[i] = (prev == pub_pieces[i] - 1);
        any |= s_lastv[i] != 0;
        if (prev >= pub_pieces[i]) report(kDevTimeoutSplitK);  // a counter left non-zero earlier
      }
      if (any) __threadfence();
    }
    consumer_sync();
    for (int i = 0; i < npub; ++i) {
      if (!s_lastv[i]) continue;
      const int rt = pub_rt[i];
      if (threadIdx.x < kRows) {
        const int64_t n = (int64_t)rt * kRows + threadIdx.x;
        float v = sum_partials(p.ws + (int64_t)rt * p.maxp * kRows + threadIdx.x, kRows, pub_pieces[i]);
        if (n < p.N) {
          if (p.bias) v = round_to(v, p.y_t) + load_as_f32(p.bias, n, p.bias_t);
          store_from_f32(p.y, n, p.y_t, v);
        }
      }
      if (threadIdx.x == 0) p.counters[rt] = 0;
    }
  }
}

// ---- host side --------------------------------------------------------------------------------
struct GemvPlan {
  int mode, ksplit, groups_per_split, ctas_n, stages, stage_bytes, sc_off, zc_off, act_off,
      seg_off, bar_off, sk, smem, items;
  // M = 1 stream-K (mode kM1)
  int units, spr, maxp, grid, ctas_per_sm, dyn = 0, clu = 0, gpc = 0, pre = 0, bf_off = 0;
  int64_t ws_floats;  // split-K / stream-K partials (0: none)
};

constexpr int kM1 = 3;
// M = 1 shared-memory tail: 2 x kMaxStages mbarriers, the abort flag, two stage tags per stage,
// the "activations staged" mbarrier.
constexpr int kM1Tail = 8 * 2 * kMaxStages + 16 + 8 * kMaxStages + 8;
// Prebuilt B fragments of one 128-k group: 8 slices x 32 lanes x 8 bytes.
constexpr int kBfGroupBytes = 8 * 32 * 8;

// CTA that owns unit u when `units` units are split evenly over `grid` CTAs (host copy).
static int owner_of(int64_t u, int64_t units, int64_t grid) { return (int)(((u + 1) * grid - 1) / units); }

// The M = 1 stream-K plan, when the whole activation row fits the shared-memory budget.
static bool plan_m1(const Weight& w, GemvPlan& pl) {
  if (w.desc.bits != 4 || w.desc.block_size > 128) return false;
  const int G = 128, seg = w.desc.block_size;
  const int gps = w.gv_gps;
  if (gps != std::min(4, seg / 16)) return false;  // the handle's boxes follow the same rule
  const int st = dtype_size(w.desc.dequant_dtype);
  const int sc_bytes = (kScaleRows * w.gv_nbs * st + 127) / 128 * 128;
  pl.sc_off = gps * kRows * 64;
  pl.zc_off = pl.sc_off + sc_bytes;
  pl.stage_bytes = (pl.zc_off + (w.zps.ptr ? sc_bytes : 0) + 1023) / 1024 * 1024;
  const int kr = (int)w.groups * G;
  const int act_bytes = (kr * 2 + 15) / 16 * 16;
  const int seg_bytes = (kr / seg) * 16;
  const int fixed = act_bytes + seg_bytes + kM1Tail;
  // Shared memory: the ring, the staged activations, the segment factors, the prebuilt B
  // fragments of `bf_groups` groups, then barriers, the abort flag and the stage tags.
  auto layout = [&](int stages, int bf_groups) {
    pl.stages = stages;
    pl.act_off = stages * pl.stage_bytes;
    pl.seg_off = pl.act_off + act_bytes;
    pl.bf_off = pl.seg_off + seg_bytes;
    pl.bar_off = pl.bf_off + bf_groups * kBfGroupBytes;
    pl.smem = pl.bar_off + kM1Tail;
  };
  // the most stages that fit with `extra` bytes of fragments
  auto stages_with = [&](int extra) { return std::min(kMaxStages, (kSmemBudget - fixed - extra) / pl.stage_bytes); };
  int stages = stages_with(0);
  pl.ctas_per_sm = 2;
  if (stages < 2) return false;
  pl.mode = kM1;
  layout(stages, 0);
  pl.sk = kr + 16;
  pl.ctas_n = (int)(w.n_pad / kRows);
  pl.spr = (int)w.groups;
  pl.units = pl.ctas_n * pl.spr;  // one unit = 128 rows x one 64-byte group
  pl.grid = std::min(pl.units, pl.ctas_per_sm * w.num_sms);
  pl.ksplit = 1;
  pl.groups_per_split = (int)w.groups;
  pl.items = pl.ctas_n;
  pl.maxp = 1;
  for (int rt = 0; rt < pl.ctas_n; ++rt) {
    const int pieces = owner_of((int64_t)rt * pl.spr + pl.spr - 1, pl.units, pl.grid) -
                       owner_of((int64_t)rt * pl.spr, pl.units, pl.grid) + 1;
    pl.maxp = std::max(pl.maxp, pieces);
  }
  pl.ws_floats = pl.maxp > 1 ? (int64_t)pl.ctas_n * pl.maxp * kRows : 0;
  // Prebuilt fragments (hand-out mode) when they leave the ring at least three stages (or all
  // it had). The other modes use each fragment once, so building them would only add a step.
  auto try_pre = [&](int bf_groups) {
    const int sp = stages_with(bf_groups * kBfGroupBytes);
    if (sp >= 2 && sp >= std::min(3, stages)) {
      pl.pre = 1;
      layout(sp, bf_groups);
    }
  };
  // Many row tiles per CTA (the lm_head): whole row tiles in arrival order instead of an even
  // static split, so the CTAs that get more memory bandwidth take more tiles and the call ends
  // with its CTAs together; no partial sums. Uses counters[0].
  pl.dyn = pl.ctas_n >= 2 * pl.grid;
  if (pl.dyn) {
    pl.maxp = 1;
    pl.ws_floats = 0;
    try_pre((int)w.groups);
    return true;
  }
  // Few row tiles (decode-sized calls): a row tile's K split over a cluster of up to 8 CTAs whose
  // whole shares fit their rings (all copies issued at once, before the previous kernel ends),
  // partial sums reduced in distributed shared memory. The smallest cluster that gives every SM
  // a CTA; else the largest that fits.
  int best = 0;
  for (int ks = 1; ks <= 8; ks *= 2) {
    const int gpc = (int)((w.groups + ks - 1) / ks);
    const int need = (gpc + gps - 1) / gps;
    if (need > kMaxStages || need * pl.stage_bytes + fixed > kSmemBudget) continue;
    if ((int64_t)pl.ctas_n * ks > (int64_t)pl.ctas_per_sm * w.num_sms) break;
    best = ks;
    if (pl.ctas_n * ks >= w.num_sms) break;
  }
  if (best > 0) {
    pl.clu = best;
    pl.gpc = (int)((w.groups + best - 1) / best);
    const int need = std::max(1, (pl.gpc + gps - 1) / gps);
    layout(need, 0);
    pl.grid = pl.ctas_n * best;
    pl.maxp = 1;
    pl.ws_floats = 0;
    return true;
  }
  return true;
}

static int seg_of(const Weight& w) {
  const int G = 512 / w.desc.bits;
  return std::min<int>(std::min(w.desc.block_size, G), 128);
}

// Groups per stage and scale blocks per stage of a handle (fixed at creation: the TMA boxes).
void gemv_stage_shape(const Weight& w, int* gps, int* nbs) {
  const int G = 512 / w.desc.bits;
  const int spg = G / seg_of(w);  // segments per group
  *gps = std::max(1, std::min(4, 8 / spg));
  const int span = *gps * G;
  *nbs = w.desc.block_size <= span ? span / w.desc.block_size : 1;
}

static GemvPlan plan_gemv(const Weight& w, int64_t m) {
  GemvPlan pl{};
  if (m == 1 && plan_m1(w, pl)) return pl;
  pl = GemvPlan{};
  const int G = 512 / w.desc.bits;
  const int seg = seg_of(w);
  const int spg = G / seg;
  const int gps = w.gv_gps;
  pl.mode = (m == 1 && spg * gps <= 8) ? kCols : (m <= 8 ? kSegMT1 : kSegMT2);
  const int mp = pl.mode == kCols ? 1 : (pl.mode == kSegMT1 ? 8 : 16);
  pl.ctas_n = (int)(w.n_pad / kRows);
  const int64_t groups = w.groups;
  const int target = 2 * w.num_sms;
  // split K for parallelism (enough items for every CTA) and for the activation staging to fit
  int ksplit = 1;
  if (pl.ctas_n < target) ksplit = (int)std::min<int64_t>((target + pl.ctas_n - 1) / pl.ctas_n, groups);
  const int st = dtype_size(w.desc.dequant_dtype);
  const int w_bytes = gps * kRows * 64;
  const int sc_bytes = (kScaleRows * w.gv_nbs * st + 127) / 128 * 128;
  pl.sc_off = w_bytes;
  pl.zc_off = pl.sc_off + sc_bytes;
  pl.stage_bytes = (pl.zc_off + (w.zps.ptr ? sc_bytes : 0) + 1023) / 1024 * 1024;
  for (;;) {
    // whole stages per item: a stage then never straddles the blocks of its scale box
    const int gps_split = (int)(((groups + ksplit - 1) / ksplit + gps - 1) / gps * gps);
    const int kr = gps_split * G;
    pl.sk = kr + 16;
    const int act_bytes = ((mp == 1 ? kr : mp * pl.sk) * 2 + 15) / 16 * 16;
    const int seg_bytes = (kr / seg) * mp * 16;
    const int fixed = act_bytes + seg_bytes + 8 * 2 * kMaxStages + 16;
    const int stages = std::min(kMaxStages, (kSmemBudget - fixed) / pl.stage_bytes);
    if (stages >= 2 || gps_split <= gps) {
      pl.groups_per_split = gps_split;
      pl.stages = std::max(2, stages);
      pl.act_off = pl.stages * pl.stage_bytes;
      pl.seg_off = pl.act_off + act_bytes;
      pl.bar_off = pl.seg_off + seg_bytes;
      pl.smem = pl.bar_off + 8 * 2 * kMaxStages + 16;
      break;
    }
    ++ksplit;
  }
  pl.ksplit = (int)((groups + pl.groups_per_split - 1) / pl.groups_per_split);
  pl.items = pl.ctas_n * pl.ksplit;
  pl.grid = std::min(pl.items, 2 * w.num_sms);
  pl.ws_floats = pl.ksplit > 1 ? (int64_t)pl.ksplit * m * w.n_pad : 0;
  return pl;
}

template <tq4_dtype AT, int SPS, bool HOLD>
static cudaError_t launch_m1_t(const Weight& w, const GemvArgs& args, int grid, int smem, cudaStream_t st) {
  auto kern = gemv_m1_kernel<AT, SPS, HOLD>;
  static std::atomic<uint64_t> attr_set{0};  // per device, once per instantiation
  {
    const cudaError_t e = set_smem_limit_once(kern, kSmemBudget + 1024, attr_set);
    if (e != cudaSuccess) return e;
  }
  if (args.clu > 1) {  // a thread-block cluster of args.clu CTAs along x, plus the dependent launch
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem + 1024;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = args.clu;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, w.gv_wmap, w.gv_smap, w.gv_zmap, args);
  }
  return launch_pdl(kern, dim3(grid), dim3(kGemvThreads), smem + 1024, st, w.gv_wmap, w.gv_smap, w.gv_zmap,
                    args);
}

template <tq4_dtype AT, bool HOLD>
static cudaError_t launch_m1_hold(const Weight& w, const GemvArgs& args, int grid, int smem, cudaStream_t st) {
  switch (std::min<int>(w.desc.block_size, 128) / 16) {
    case 1: return launch_m1_t<AT, 1, HOLD>(w, args, grid, smem, st);
    case 2: return launch_m1_t<AT, 2, HOLD>(w, args, grid, smem, st);
    case 4: return launch_m1_t<AT, 4, HOLD>(w, args, grid, smem, st);
    default: return launch_m1_t<AT, 8, HOLD>(w, args, grid, smem, st);
  }
}

template <tq4_dtype AT>
static cudaError_t launch_m1_sps(const Weight& w, const GemvArgs& args, int grid, int smem, cudaStream_t st) {
  if (args.dyn || args.clu) return launch_m1_hold<AT, false>(w, args, grid, smem, st);
  return launch_m1_hold<AT, true>(w, args, grid, smem, st);
}

template <int BITS, tq4_dtype AT, int MODE>
static cudaError_t launch_gemv_t(const Weight& w, const GemvArgs& args, int smem, cudaStream_t st) {
  auto kern = gemv_kernel<BITS, AT, MODE>;
  static std::atomic<uint64_t> attr_set{0};  // per device, once per instantiation
  {
    const cudaError_t e = set_smem_limit_once(kern, kSmemBudget + 1024, attr_set);
    if (e != cudaSuccess) return e;
  }
  const int grid = std::min(args.items, 2 * w.num_sms);
  kern<<<grid, kGemvThreads, smem + 1024, st>>>(w.gv_wmap, w.gv_smap, w.gv_zmap, args);
  return cudaGetLastError();
}

template <int BITS, tq4_dtype AT>
static cudaError_t launch_gemv_mode(const Weight& w, const GemvArgs& args, int mode, int smem,
                                    cudaStream_t st) {
  switch (mode) {
    case kCols: return launch_gemv_t<BITS, AT, kCols>(w, args, smem, st);
    case kSegMT1: return launch_gemv_t<BITS, AT, kSegMT1>(w, args, smem, st);
    default: return launch_gemv_t<BITS, AT, kSegMT2>(w, args, smem, st);
  }
}

template <int BITS>
static cudaError_t launch_gemv_bits(const Weight& w, const GemvArgs& args, tq4_dtype a_t, int mode,
                                    int smem, cudaStream_t st) {
  switch (a_t) {
    case TQ4_F16: return launch_gemv_mode<BITS, TQ4_F16>(w, args, mode, smem, st);
    case TQ4_BF16: return launch_gemv_mode<BITS, TQ4_BF16>(w, args, mode, smem, st);
    default: return launch_gemv_mode<BITS, TQ4_F32>(w, args, mode, smem, st);
  }
}

// The GEMV's TMA descriptors of a new handle: one 128-row x 64-byte box of packed rows, and
// 136-row x (blocks of a stage) boxes of the block-major scales / zero points.
tq4_status make_gemv_maps(Weight& w) {
  w.gv_maps_ok = false;
  gemv_stage_shape(w, &w.gv_gps, &w.gv_nbs);
  const int st = dtype_size(w.desc.dequant_dtype);
  const CUtensorMapDataType sdt = st == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  TQ4_TRY(make_map(&w.gv_wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q.ptr, w.row_bytes, w.n_pad,
                   w.row_bytes, 64, kRows, CU_TENSOR_MAP_SWIZZLE_NONE));
  TQ4_TRY(make_map(&w.gv_smap, sdt, w.scales.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, kScaleRows,
                   w.gv_nbs, CU_TENSOR_MAP_SWIZZLE_NONE));
  if (w.zps.ptr)
    TQ4_TRY(make_map(&w.gv_zmap, sdt, w.zps.ptr, w.n_pad, w.blocks_pad, w.n_pad * st, kScaleRows,
                     w.gv_nbs, CU_TENSOR_MAP_SWIZZLE_NONE));
  else
    w.gv_zmap = w.gv_smap;  // never loaded
  w.gv_maps_ok = true;
  return TQ4_OK;
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

// A staging transform of the decoder's fused projections (GemvArgs::pro).
struct GemvPrologue {
  int mode;
  const float* w;
  const float* b;
  float eps;
};

static tq4_status gemv_launch(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                              tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st, float* ws,
                              int* counters, int64_t ws_capacity_floats, int64_t ctr_capacity,
                              const GemvPrologue* pro);

tq4_status run_gemv_with(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                         tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st,
                         float* ws, int* counters, int64_t ws_capacity_floats, int64_t ctr_capacity) {
  return gemv_launch(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st, ws, counters, ws_capacity_floats, ctr_capacity,
                     nullptr);
}

static tq4_status gemv_launch(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                              tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st, float* ws,
                              int* counters, int64_t ws_capacity_floats, int64_t ctr_capacity,
                              const GemvPrologue* pro) {
  if (!w.gv_maps_ok) {
    set_error("GEMV: the handle has no TMA descriptors");
    return TQ4_ERR_CUDA;
  }
  if (m == 1 && rows_eligible(w) && (!pro || (pro->mode <= 1 && rows_slices(w) == 1))) {
    // one activation row: the 32-row-unit kernel (gemv_rows.cu), K-sliced for rows of more than
    // 8 packed groups, with the RMSNorm prologue of the decoder's fused projections when asked (the
    // decoder's other projections keep the 128-row kernel: measured faster within its step)
    if (counters == nullptr || ctr_capacity < rows_counters(w) ||
        (rows_ws_floats(w) > 0 && (ws == nullptr || ws_capacity_floats < rows_ws_floats(w)))) {
      set_error("GEMV: the unit hand-out needs %lld counters and %lld workspace floats",
                (long long)rows_counters(w), (long long)rows_ws_floats(w));
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    RowsDst dst;
    dst.y[0] = y;
    RowsNorm norm;
    if (pro && pro->mode == 1) {
      norm.w = pro->w;
      norm.eps = pro->eps;
    }
    return run_gemv_rows(w, a, a_t, bias, bias_t, y_t, dst, counters, st, pro && pro->mode == 1 ? &norm : nullptr, ws);
  }
  const GemvPlan pl = plan_gemv(w, m);
  GemvArgs args{};
  args.a = a;
  args.bias = bias;
  args.bias_t = bias_t;
  args.y = y;
  args.y_t = y_t;
  args.ldy = ldy;
  args.z_const = w.z_const;
  args.has_zp = w.zps.ptr != nullptr;
  args.st_bytes = dtype_size(w.desc.dequant_dtype);
  args.st_bf16 = w.desc.dequant_dtype == TQ4_BF16;
  args.K = (int)w.desc.K;
  args.N = (int)w.desc.N;
  args.M = (int)m;
  args.bs_log2 = w.bs_log2;
  int seg_log2 = 0;
  while ((1 << seg_log2) < seg_of(w)) ++seg_log2;
  args.seg_log2 = seg_log2;
  args.groups = (int)w.groups;
  args.groups_per_split = pl.groups_per_split;
  args.gps = w.gv_gps;
  args.nbs = w.gv_nbs;
  args.stages = pl.stages;
  args.stage_bytes = pl.stage_bytes;
  args.sc_off = pl.sc_off;
  args.zc_off = pl.zc_off;
  args.act_off = pl.act_off;
  args.seg_off = pl.seg_off;
  args.bar_off = pl.bar_off;
  args.sk = pl.sk;
  args.ctas_n = pl.ctas_n;
  args.ksplit = pl.ksplit;
  args.items = pl.items;
  args.units = pl.units;
  args.spr = pl.spr;
  args.maxp = pl.maxp;
  args.dyn = pl.dyn;
  args.pre = pl.pre;
  args.bf_off = pl.bf_off;
  args.clu = pl.clu;
  args.gpc = pl.gpc;
  if (pro && pro->mode) {
    if (pl.mode != kM1 || m != 1 || a_t != TQ4_F32) {
      set_error("fused projection: needs M = 1, f32 activations and a 4-bit weight with block <= 128");
      return TQ4_ERR_UNSUPPORTED;
    }
    args.pro = pro->mode;
    args.pro_w = pro->w;
    args.pro_b = pro->b;
    args.pro_eps = pro->eps;
  }
  args.n_pad = w.n_pad;
  const int nctr = pl.dyn ? 1 : (pl.ws_floats > 0 ? pl.ctas_n : 0);
  if (pl.ws_floats > 0 || nctr > 0) {
    if ((pl.ws_floats > 0 && (ws == nullptr || pl.ws_floats > ws_capacity_floats)) || counters == nullptr ||
        nctr > ctr_capacity) {
      set_error("split-K workspace too small: need %lld floats and %d counters",
                (long long)pl.ws_floats, nctr);
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    args.ws = ws;
    args.counters = counters;
  }
  cudaError_t e;
  if (pl.mode == kM1) {
    switch (a_t) {
      case TQ4_F16: e = launch_m1_sps<TQ4_F16>(w, args, pl.grid, pl.smem, st); break;
      case TQ4_BF16: e = launch_m1_sps<TQ4_BF16>(w, args, pl.grid, pl.smem, st); break;
      default: e = launch_m1_sps<TQ4_F32>(w, args, pl.grid, pl.smem, st); break;
    }
  } else if (w.desc.bits == 4) e = launch_gemv_bits<4>(w, args, a_t, pl.mode, pl.smem, st);
  else if (w.desc.bits == 2) e = launch_gemv_bits<2>(w, args, a_t, pl.mode, pl.smem, st);
  else e = launch_gemv_bits<8>(w, args, a_t, pl.mode, pl.smem, st);
  if (e != cudaSuccess) {
    set_error("GEMV launch failed: %s", cudaGetErrorString(e));
    return TQ4_ERR_CUDA;
  }
  return TQ4_OK;
}

// Workspace of a plain call (tq4_matmul, tq4_matmul_noalloc): partial-sum floats and counters.
int64_t gemv_workspace_floats(const Weight& w, int64_t m) {
  if (m == 1 && rows_eligible(w)) return rows_ws_floats(w);
  return plan_gemv(w, m).ws_floats;
}

// Counters a call of the 128-row kernels uses (zero-initialised, left at zero by the kernel): one
// per row tile for split partial sums, one for the M = 1 row-tile hand-out, none otherwise.
static int64_t tile_counter_count(const Weight& w, int64_t m) {
  const GemvPlan pl = plan_gemv(w, m);
  return pl.dyn ? 1 : (pl.ws_floats > 0 ? pl.ctas_n : 0);
}

// The decoder's fused projection (include/tq4_decoder.h, tq4_matmul_fused).
tq4_status run_gemv_fused(const Weight& w, const float* x, const float* x2, const float* norm_w, float eps,
                          int mode, const float* residual, float* y, cudaStream_t st) {
  float* ws = nullptr;
  int* ctr = nullptr;
  // the 32-row-unit kernel takes plain calls and the RMSNorm prologue on rows of at most 8 groups;
  // SwiGLU and longer rows run in the 128-row kernel
  const bool plain = mode <= 1 && rows_eligible(w) && rows_slices(w) == 1;
  const int64_t need = plain ? 0 : plan_gemv(w, 1).ws_floats;
  const int64_t nctr = plain ? 1 : tile_counter_count(w, 1);
  if (need > 0 || nctr > 0) TQ4_TRY(gemv_workspace(w, st, need * 4, nctr, &ws, &ctr));
  GemvPrologue pro{mode, norm_w, x2, eps};
  return gemv_launch(w, x, 1, TQ4_F32, residual, TQ4_F32, y, TQ4_F32, w.desc.N, st, ws, ctr, need, nctr, &pro);
}

// Counters a plain call uses (zero-initialised, left at zero by the kernel): the unit hand-out of
// the 32-row-unit kernel, or those of the 128-row kernels.
int64_t gemv_counter_count(const Weight& w, int64_t m) {
  if (m == 1 && rows_eligible(w)) return rows_counters(w);
  return tile_counter_count(w, m);
}

tq4_status run_gemv(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                    tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  float* ws = nullptr;
  int* ctr = nullptr;
  const int64_t need = gemv_workspace_floats(w, m);
  const int64_t nctr = gemv_counter_count(w, m);
  if (need > 0 || nctr > 0) TQ4_TRY(gemv_workspace(w, st, need * 4, nctr, &ws, &ctr));
  return run_gemv_with(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st, ws, ctr, need, nctr);
}

}  // namespace tq4
