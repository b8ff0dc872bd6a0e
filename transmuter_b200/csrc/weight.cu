// Weight preparation (the load-time half of the operator) and the bit-exact dequantize.
//
// tq4_weight_create copies B, scales and zero points to the device once and rewrites them into
// the handle's layout (common.cuh): B as 64-byte groups per row in fragment order, scales and
// zero points as [N_pad][blocks_pad] arrays in the dequantize type T. The reference does the
// same work once per weight in Transmuter.move/2 (lib/transmuter.ex:1155-1164,1230-1240).
#include "internal.cuh"

namespace tq4 {

__device__ int32_t g_device_status = 0;
__device__ long long g_wait_cycles = 2000000000LL;  // about one second at the B200's clocks

// One thread per output 32-bit word of the packed layout: gathers its 32/BITS elements from
// the raw rows (element k of row n = bits [(k%per)*BITS, ...) of byte k/per, packed.ex:11-23).
// `flip` is 2^(BITS-1) for signed data, 0 otherwise: a signed value v (sign extended,
// quantized.ex:294-300) is stored as u = v + 2^(BITS-1), which is the raw bits with the top bit
// flipped, and its zero point is raised by the same amount, so q - z is unchanged.
template <int BITS>
__global__ void repack_kernel(const uint8_t* __restrict__ raw, int64_t raw_row_bytes,
                              int64_t n_rows, int64_t k_valid, uint32_t* __restrict__ out,
                              int64_t row_bytes, int64_t n_pad, uint32_t flip) {
  constexpr int PER = 8 / BITS;
  constexpr int MASK = (1 << BITS) - 1;
  const int64_t words_per_row = row_bytes / 4;
  const int64_t total = n_pad * words_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / words_per_row;
    const int64_t wbyte = (i % words_per_row) * 4;  // byte offset of this word in the row
    uint32_t word = 0;
    if (n < n_rows) {
      // Invert packed_position: every element slot of this word -> its k.
      const int64_t c = wbyte / 64;
      const int rem = (int)(wbyte % 64);
      const int t = rem / 16, w = (rem % 16) / 4;
      for (int slot = 0; slot < 32 / BITS; ++slot) {
        int j, e;
        if (BITS == 4) {
          const int pos = slot;  // nibble position 0..7
          e = (pos / 4) + 2 * (pos % 2);
          j = 2 * w + (pos % 4) / 2;
        } else if (BITS == 2) {
          const int pos = slot;  // 2-bit position 0..15
          const int pp = pos % 8;
          e = (pos / 8) + 2 * (pp % 2);
          j = 4 * w + pp / 2;
        } else {
          e = slot;
          j = w;
        }
        const int64_t k = c * (512 / BITS) + 16 * j + 4 * t + e;
        if (k < k_valid) {
          const uint8_t byte = raw[n * raw_row_bytes + k / PER];
          const uint32_t v = ((byte >> ((k % PER) * BITS)) & MASK) ^ flip;
          word |= v << (slot * BITS);
        }
      }
    }
    out[i] = word;
  }
}

// scales / float zero points [N][blocks] of type `src_t` -> [blocks_pad][n_pad] (block-major, so
// a run of rows of one block is contiguous) in T with one rounding (Nx.as_type,
// quantized.ex:237 and :314). Padding entries are 0.
template <typename T>
__global__ void convert_blocks_kernel(const void* __restrict__ src, tq4_dtype src_t, int64_t n,
                                      int64_t blocks, T* __restrict__ dst, int64_t n_pad,
                                      int64_t blocks_pad) {
  const int64_t total = n_pad * blocks_pad;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / n_pad, r = i % n_pad;
    float v = 0.f;
    if (r < n && b < blocks) v = load_as_f32(src, r * blocks + b, src_t);
    dst[i] = from_f32<T>(v);
  }
}

// Packed zero points: row r holds ceil(blocks*bits/8) bytes (the reshape to {N, :auto} of
// quantized.ex:316-322); value b of the row is unpacked like B (sign extended when the zero
// points are s8), raised by `offset` (2^(bits-1) for signed data, see repack_kernel) and cast to
// T (exact), stored block-major like the scales.
template <typename T>
__global__ void unpack_zp_kernel(const uint8_t* __restrict__ zp, int64_t zp_row_bytes, int bits,
                                 int64_t n, int64_t blocks, T* __restrict__ dst, int64_t n_pad,
                                 int64_t blocks_pad, int zp_signed, float offset) {
  const int per = 8 / bits, mask = (1 << bits) - 1;
  const int64_t total = n_pad * blocks_pad;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / n_pad, r = i % n_pad;
    float v = 0.f;
    if (r < n && b < blocks) {
      const uint8_t byte = zp[r * zp_row_bytes + b / per];
      int q = (byte >> ((b % per) * bits)) & mask;
      if (zp_signed && q >= (1 << (bits - 1))) q -= 1 << bits;
      v = (float)q + offset;
    }
    dst[i] = from_f32<T>(v);
  }
}

// ---- dequantize_weight/4 (quantized.ex:234-240), bit-exact -----------------------------------
// W[n][k] = RN_T( RN_T(q - z) * s ) for k < K. The subtraction is done in double (exact for
// q < 256 and any zero point of T with an exponent gap below 2^45) and rounded once to T; the
// product of two T values is exact in f32 for f16/bf16, and __fmul_rn for f32.
template <int BITS, typename T>
__device__ __forceinline__ T dequant_one(uint32_t q, float z, float s) {
  if constexpr (sizeof(T) == 4) {
    const float d = __fsub_rn((float)q, z);
    return __fmul_rn(d, s);
  } else {
    const double d64 = (double)q - (double)z;
    float d;
    if constexpr (std::is_same<T, __half>::value) d = __half2float(__double2half(d64));
    else d = __bfloat162float(__double2bfloat16(d64));
    return from_f32<T>(d * s);  // exact product, one rounding
  }
}

template <int BITS, typename T>
__global__ void dequant_kernel(const uint8_t* __restrict__ q, int64_t row_bytes,
                               const T* __restrict__ scales, const T* __restrict__ zps,
                               float z_const, int64_t n_pad, int bs_log2, int64_t n,
                               int64_t k, const int64_t* __restrict__ rows, int64_t n_rows,
                               T* __restrict__ out) {
  pdl_wait();  // row indices may come from the previous kernel
  pdl_trigger();
  const int64_t total = n * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r_out = i / k, kk = i % k;
    const int64_t r = rows ? rows[r_out] : r_out;
    if (r < 0 || r >= n_rows) {  // an index outside the table: report it, never read it
      report(kDevBadArgument);
      out[i] = from_f32<T>(0.f);
      continue;
    }
    int64_t byte;
    int shift;
    packed_position<BITS>(kk, byte, shift);
    const uint32_t v = (q[r * row_bytes + byte] >> shift) & ((1u << BITS) - 1);
    const int64_t b = kk >> bs_log2;
    const float s = to_f32(scales[b * n_pad + r]);
    const float z = zps ? to_f32(zps[b * n_pad + r]) : z_const;
    out[i] = dequant_one<BITS, T>(v, z, s);
  }
}

// ---- host side --------------------------------------------------------------------------------
static int grid_for(int64_t total, int threads) {
  int64_t g = (total + threads - 1) / threads;
  return (int)std::min<int64_t>(std::max<int64_t>(g, 1), 148 * 32);
}

template <typename T>
static void launch_convert(const Weight& w, const void* src, tq4_dtype src_t, T* dst, cudaStream_t st) {
  const int64_t total = w.n_pad * w.blocks_pad;
  convert_blocks_kernel<T><<<grid_for(total, 256), 256, 0, st>>>(src, src_t, w.desc.N, w.blocks,
                                                                   dst, w.n_pad, w.blocks_pad);
}

template <typename T>
static void launch_unpack_zp(const Weight& w, const uint8_t* zp, T* dst, cudaStream_t st) {
  const int64_t total = w.n_pad * w.blocks_pad;
  const int64_t zp_row = (w.blocks * w.desc.bits + 7) / 8;
  const float offset = w.desc.b_signed ? (float)(1 << (w.desc.bits - 1)) : 0.f;
  unpack_zp_kernel<T><<<grid_for(total, 256), 256, 0, st>>>(zp, zp_row, w.desc.bits, w.desc.N, w.blocks, dst,
                                                              w.n_pad, w.blocks_pad, w.desc.zp_dtype == TQ4_S8,
                                                              offset);
}

// Per-row bound of the f32 weights: wexp[n] with max_b |s_b| * max(|z_b|, |2^bits - 1 - z_b|) <= 2^wexp[n]
// (frexp exponent of that maximum; 0 for an all-zero or non-finite row).
__global__ void row_exponent_kernel(const float* __restrict__ scales, const float* __restrict__ zps, float z_const,
                                    int64_t blocks, int64_t n, int64_t n_pad, float qmax, int32_t* __restrict__ out) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n_pad; r += (int64_t)gridDim.x * blockDim.x) {
    float mx = 0.f;
    if (r < n) {
      for (int64_t b = 0; b < blocks; ++b) {
        const float s = fabsf(scales[b * n_pad + r]);
        const float z = zps ? zps[b * n_pad + r] : z_const;
        mx = fmaxf(mx, s * fmaxf(fabsf(z), fabsf(qmax - z)));
      }
    }
    int e = 0;
    if (mx > 0.f && isfinite(mx)) frexpf(mx, &e);
    out[r] = e;
  }
}

// The GEMM's f16 block scales of f32 weights: s * 2^-wexp[n] rounded once to f16.
__global__ void scale16_kernel(const float* __restrict__ scales, const int32_t* __restrict__ wexp,
                               int64_t n_pad, int64_t total, __half* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(ldexpf(scales[i], -wexp[i % n_pad]));
}

tq4_status prepare_weight(Weight& w, const Source& b_src, const Source& s_src, const Source* zp_src) {
  const tq4_weight_desc& d = w.desc;
  cudaStream_t st = w.stream;
  const int64_t raw_row = w.blocks * d.block_size * d.bits / 8;
  const int64_t b_bytes = d.N * raw_row;
  const int64_t s_bytes = d.N * w.blocks * dtype_size(d.scale_dtype);
  int64_t zp_bytes = 0;
  if (d.zp_kind == TQ4_ZP_PACKED) zp_bytes = d.N * ((w.blocks * d.bits + 7) / 8);
  if (d.zp_kind == TQ4_ZP_FLOAT) zp_bytes = d.N * w.blocks * dtype_size(d.zp_dtype);

  // Staging copies of the raw inputs: memory (host or device) or file ranges.
  if (b_src.length != b_bytes || s_src.length != s_bytes || (zp_src ? zp_src->length : 0) != zp_bytes) {
    set_error("MatMulNBits: input sizes do not match the description");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceBuffer raw_b, raw_s, raw_z;
  TQ4_TRY(raw_b.alloc(b_bytes));
  TQ4_TRY(raw_s.alloc(s_bytes));
  if (zp_bytes) TQ4_TRY(raw_z.alloc(zp_bytes));
  TQ4_TRY(fill_device(raw_b.ptr, b_src, w.device, st));
  TQ4_TRY(fill_device(raw_s.ptr, s_src, w.device, st));
  if (zp_bytes) TQ4_TRY(fill_device(raw_z.ptr, *zp_src, w.device, st));

  const int64_t words = w.n_pad * w.row_bytes / 4;
  const int grid = grid_for(words, 256);
  const int64_t k_valid = w.blocks * d.block_size;
  uint32_t* qdst = static_cast<uint32_t*>(w.q.ptr);
  const uint8_t* rb = static_cast<const uint8_t*>(raw_b.ptr);
  const uint32_t flip = d.b_signed ? 1u << (d.bits - 1) : 0u;
  if (d.bits == 4) repack_kernel<4><<<grid, 256, 0, st>>>(rb, raw_row, d.N, k_valid, qdst, w.row_bytes, w.n_pad, flip);
  else if (d.bits == 2) repack_kernel<2><<<grid, 256, 0, st>>>(rb, raw_row, d.N, k_valid, qdst, w.row_bytes, w.n_pad, flip);
  else repack_kernel<8><<<grid, 256, 0, st>>>(rb, raw_row, d.N, k_valid, qdst, w.row_bytes, w.n_pad, flip);
  TQ4_CUDA(cudaGetLastError());

  switch (d.dequant_dtype) {
    case TQ4_F32:
      launch_convert<float>(w, raw_s.ptr, d.scale_dtype, static_cast<float*>(w.scales.ptr), st);
      if (d.zp_kind == TQ4_ZP_FLOAT) launch_convert<float>(w, raw_z.ptr, d.zp_dtype, static_cast<float*>(w.zps.ptr), st);
      if (d.zp_kind == TQ4_ZP_PACKED) launch_unpack_zp<float>(w, static_cast<const uint8_t*>(raw_z.ptr), static_cast<float*>(w.zps.ptr), st);
      break;
    case TQ4_F16:
      launch_convert<__half>(w, raw_s.ptr, d.scale_dtype, static_cast<__half*>(w.scales.ptr), st);
      if (d.zp_kind == TQ4_ZP_FLOAT) launch_convert<__half>(w, raw_z.ptr, d.zp_dtype, static_cast<__half*>(w.zps.ptr), st);
      if (d.zp_kind == TQ4_ZP_PACKED) launch_unpack_zp<__half>(w, static_cast<const uint8_t*>(raw_z.ptr), static_cast<__half*>(w.zps.ptr), st);
      break;
    default:
      launch_convert<__nv_bfloat16>(w, raw_s.ptr, d.scale_dtype, static_cast<__nv_bfloat16*>(w.scales.ptr), st);
      if (d.zp_kind == TQ4_ZP_FLOAT) launch_convert<__nv_bfloat16>(w, raw_z.ptr, d.zp_dtype, static_cast<__nv_bfloat16*>(w.zps.ptr), st);
      if (d.zp_kind == TQ4_ZP_PACKED) launch_unpack_zp<__nv_bfloat16>(w, static_cast<const uint8_t*>(raw_z.ptr), static_cast<__nv_bfloat16*>(w.zps.ptr), st);
      break;
  }
  TQ4_CUDA(cudaGetLastError());
  if (d.dequant_dtype == TQ4_F32) {  // the tensor-core GEMM's f16 form of f32 weights
    TQ4_TRY(w.wexp.alloc(w.n_pad * 4));
    row_exponent_kernel<<<grid_for(w.n_pad, 256), 256, 0, st>>>(
        static_cast<const float*>(w.scales.ptr), static_cast<const float*>(w.zps.ptr), w.z_const, w.blocks,
        d.N, w.n_pad, (float)((1 << d.bits) - 1), static_cast<int32_t*>(w.wexp.ptr));
    TQ4_CUDA(cudaGetLastError());
    if (d.zp_kind == TQ4_ZP_NONE) {
      const int64_t total = w.n_pad * w.blocks_pad;
      TQ4_TRY(w.scales16.alloc(total * 2));
      scale16_kernel<<<grid_for(total, 256), 256, 0, st>>>(static_cast<const float*>(w.scales.ptr),
                                                            static_cast<const int32_t*>(w.wexp.ptr), w.n_pad,
                                                            total, static_cast<__half*>(w.scales16.ptr));
      TQ4_CUDA(cudaGetLastError());
    }
  }
  // The staging buffers are freed when this function returns; finish the kernels first.
  TQ4_CUDA(cudaStreamSynchronize(st));
  return TQ4_OK;
}

// Fusion.matmuls/2 for packed weights (lib/transmuter/fusion.ex:430-540): the rows of parts[0],
// then parts[1], ... copied into w's buffers (already laid out for the summed N, zero-filled by the
// caller where the copies do not reach). The packed rows are contiguous per part; the block-major
// scales and zero points are pitched copies (one run of N_i entries per block row). The per-row
// exponents and the f16 block scales of f32 weights derive from the scales, so they are computed
// again over the merged scales, exactly as for a handle built from the concatenated inputs.
tq4_status merge_weight(Weight& w, const Weight* const* parts, int count) {
  const tq4_weight_desc& d = w.desc;
  cudaStream_t st = w.stream;
  const int tsz = dtype_size(d.dequant_dtype);
  int64_t off = 0;
  for (int i = 0; i < count; ++i) {
    const Weight& p = *parts[i];
    const int64_t n = p.desc.N;
    TQ4_CUDA(cudaMemcpyAsync(static_cast<uint8_t*>(w.q.ptr) + off * w.row_bytes, p.q.ptr, n * w.row_bytes,
                             cudaMemcpyDeviceToDevice, st));
    TQ4_CUDA(cudaMemcpy2DAsync(static_cast<uint8_t*>(w.scales.ptr) + off * tsz, w.n_pad * tsz, p.scales.ptr,
                               p.n_pad * tsz, n * tsz, w.blocks_pad, cudaMemcpyDeviceToDevice, st));
    if (w.zps.ptr)
      TQ4_CUDA(cudaMemcpy2DAsync(static_cast<uint8_t*>(w.zps.ptr) + off * tsz, w.n_pad * tsz, p.zps.ptr,
                                 p.n_pad * tsz, n * tsz, w.blocks_pad, cudaMemcpyDeviceToDevice, st));
    off += n;
  }
  if (d.dequant_dtype == TQ4_F32) {  // the tensor-core GEMM's f16 form of f32 weights
    TQ4_TRY(w.wexp.alloc(w.n_pad * 4));
    row_exponent_kernel<<<grid_for(w.n_pad, 256), 256, 0, st>>>(
        static_cast<const float*>(w.scales.ptr), static_cast<const float*>(w.zps.ptr), w.z_const, w.blocks,
        d.N, w.n_pad, (float)((1 << d.bits) - 1), static_cast<int32_t*>(w.wexp.ptr));
    TQ4_CUDA(cudaGetLastError());
    if (d.zp_kind == TQ4_ZP_NONE) {
      const int64_t total = w.n_pad * w.blocks_pad;
      TQ4_TRY(w.scales16.alloc(total * 2));
      scale16_kernel<<<grid_for(total, 256), 256, 0, st>>>(static_cast<const float*>(w.scales.ptr),
                                                            static_cast<const int32_t*>(w.wexp.ptr), w.n_pad,
                                                            total, static_cast<__half*>(w.scales16.ptr));
      TQ4_CUDA(cudaGetLastError());
    }
  }
  TQ4_CUDA(cudaStreamSynchronize(st));
  return TQ4_OK;
}

template <int BITS, typename T>
static void launch_dequant(const Weight& w, const int64_t* rows, int64_t n_out, void* out,
                           cudaStream_t st) {
  const int64_t total = n_out * w.desc.K;
  launch_pdl(dequant_kernel<BITS, T>, dim3(grid_for(total, 256)), dim3(256), 0, st,
             static_cast<const uint8_t*>(w.q.ptr), w.row_bytes, static_cast<const T*>(w.scales.ptr),
             static_cast<const T*>(w.zps.ptr), w.z_const, w.n_pad, w.bs_log2, n_out, (int64_t)w.desc.K, rows,
             (int64_t)w.desc.N, static_cast<T*>(out));
}

template <typename T>
static void dispatch_dequant_bits(const Weight& w, const int64_t* rows, int64_t n_out, void* out,
                                  cudaStream_t st) {
  if (w.desc.bits == 4) launch_dequant<4, T>(w, rows, n_out, out, st);
  else if (w.desc.bits == 2) launch_dequant<2, T>(w, rows, n_out, out, st);
  else launch_dequant<8, T>(w, rows, n_out, out, st);
}

tq4_status run_dequant(const Weight& w, const int64_t* rows, int64_t n_out, void* out, cudaStream_t st) {
  if (n_out == 0 || w.desc.K == 0) return TQ4_OK;
  switch (w.desc.dequant_dtype) {
    case TQ4_F32: dispatch_dequant_bits<float>(w, rows, n_out, out, st); break;
    case TQ4_F16: dispatch_dequant_bits<__half>(w, rows, n_out, out, st); break;
    default: dispatch_dequant_bits<__nv_bfloat16>(w, rows, n_out, out, st); break;
  }
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

}  // namespace tq4
