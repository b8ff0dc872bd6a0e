// Shared device helpers of the tq4 kernels: float types, the device status word and bounded
// waits. Compiled for sm_100a only.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tq4.h"

namespace tq4 {

// ---- device status word ---------------------------------------------------------------------
// Kernels never trap: a bounded wait that runs out, or a device-side check that fails, writes a
// code here (first writer wins) and the kernel returns. tq4_device_status() reads and clears it.
enum DeviceCode : int32_t {
  kDevOk = 0,
  kDevTimeoutTmaFull = 0x101,     // GEMM: waited too long for a TMA stage
  kDevTimeoutStageEmpty = 0x102,  // GEMM: waited too long for the MMA to free a stage
  kDevTimeoutDequant = 0x103,     // GEMM: waited too long for the dequantized tile
  kDevTimeoutAccum = 0x104,       // GEMM: waited too long for the accumulator
  kDevTimeoutSplitK = 0x105,      // GEMV: split-K reduction counter inconsistent
  kDevTimeoutPeer = 0x106,        // sharded exchange: a peer's slice did not arrive in time
  kDevTimeoutAttn = 0x107,        // decode attention: a K/V chunk copy did not arrive in time
  kDevTimeoutStaged = 0x108,      // GEMV: waited too long for the activations to be staged
  kDevBadArgument = 0x200,
};

// Defined in weight.cu (the library is built with relocatable device code).
extern __device__ int32_t g_device_status;

__device__ __forceinline__ void report(int32_t code) { atomicCAS(&g_device_status, 0, code); }

// The limit of every bounded wait, in SM clock cycles (defined in weight.cu; about one second by
// default, set per device with tq4_set_wait_limit).
extern __device__ long long g_wait_cycles;
__device__ __forceinline__ long long wait_limit() { return *reinterpret_cast<volatile long long*>(&g_wait_cycles); }

// Programmatic dependent launch. A kernel launched with launch_pdl may start while the kernel
// before it on the stream is still running: everything it does before pdl_wait() must touch only
// memory no earlier kernel writes (weights, its own shared memory). pdl_wait() returns once the
// previous grid has completed and its writes are visible; every CTA of such a kernel passes it
// (or exits without touching global memory) so that completion stays transitive along the stream.
// pdl_trigger() lets the next kernel be scheduled; without a PDL launch both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- float types ------------------------------------------------------------------------------
template <tq4_dtype T> struct FloatOf;
template <> struct FloatOf<TQ4_F32> { using type = float; };
template <> struct FloatOf<TQ4_F16> { using type = __half; };
template <> struct FloatOf<TQ4_BF16> { using type = __nv_bfloat16; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Loads element i of a float array of runtime type t as f32.
__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, tq4_dtype t) {
  switch (t) {
    case TQ4_F16: return __half2float(static_cast<const __half*>(p)[i]);
    case TQ4_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default: return static_cast<const float*>(p)[i];
  }
}

// Element i of a scale / zero-point array stored in T (4-byte f32, or 2-byte bf16 / f16).
__device__ __forceinline__ float scale_to_f32(const void* base, int64_t i, int st_bytes, int bf) {
  if (st_bytes == 4) return static_cast<const float*>(base)[i];
  const uint16_t v = static_cast<const uint16_t*>(base)[i];
  if (bf) return __uint_as_float(((uint32_t)v) << 16);
  return __half2float(__ushort_as_half(v));
}

// One typed rounding of an f32 value that holds an exact result: the value of `x` rounded to t,
// returned as f32 (exactly representable in t).
__device__ __forceinline__ float round_to(float x, tq4_dtype t) {
  switch (t) {
    case TQ4_F16: return __half2float(__float2half_rn(x));
    case TQ4_BF16: return __bfloat162float(__float2bfloat16_rn(x));
    default: return x;
  }
}

__device__ __forceinline__ void store_from_f32(void* p, int64_t i, tq4_dtype t, float v) {
  switch (t) {
    case TQ4_F16: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
    case TQ4_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    default: static_cast<float*>(p)[i] = v; break;
  }
}

// ---- the handle's packed layout ---------------------------------------------------------------
// Each row of B is stored with a pitch of `row_bytes` (a multiple of 64) and cut into 64-byte
// groups. Group c of row n holds the elements k in [c*G, (c+1)*G), G = 64*8/bits, as four
// 16-byte pieces t = 0..3: piece t holds the elements k = c*G + 16*j + 4*t + e for the
// "steps" j = 0..G/16-1 and e = 0..3. Within a piece, the 32-bit words are laid out so that the
// magic-number conversions below yield pairs (e0, e1) and (e2, e3) of one step without shifts
// beyond one per word:
//   4 bits: word w covers steps 2w and 2w+1; nibble positions (0,4) = (step 2w, e0/e1),
//           (1,5) = (2w, e2/e3), (2,6) = (2w+1, e0/e1), (3,7) = (2w+1, e2/e3).
//   2 bits: word w covers steps 4w..4w+3; 2-bit positions (p, p+8) for p = 0..7 hold
//           (step 4w + p/2, e0/e1) for even p and (4w + p/2, e2/e3) for odd p.
//   8 bits: word w is step w, bytes e0..e3 in order.
// Padding elements (k >= blocks*block_size) and padding rows hold 0.

// Position (byte, bit shift) in a row of the packed layout of element k.
template <int BITS> __host__ __device__ __forceinline__ void packed_position(int64_t k, int64_t& byte, int& shift) {
  constexpr int G = 512 / BITS;  // elements per 64-byte group
  const int64_t c = k / G;
  const int r = (int)(k % G);
  const int j = r / 16, t = (r % 16) / 4, e = r % 4;
  if (BITS == 4) {
    const int w = j / 2, odd = j % 2;
    const int pos = (e & 1) * 4 + odd * 2 + (e >> 1);  // nibble position in the word
    byte = c * 64 + t * 16 + w * 4 + pos / 2;
    shift = (pos % 2) * 4;
  } else if (BITS == 2) {
    const int w = j / 4, sub = j % 4;
    const int p = sub * 2 + (e >> 1);                   // pair index 0..7
    const int pos = p + (e & 1) * 8;                    // 2-bit position in the word
    byte = c * 64 + t * 16 + w * 4 + pos / 4;
    shift = (pos % 4) * 2;
  } else {
    byte = c * 64 + t * 16 + j * 4 + e;
    shift = 0;
  }
}

// ---- small PTX helpers ------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t x, uint32_t mask, uint32_t magic) {
  uint32_t r;
  // (x & mask) | magic
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(x), "r"(mask), "r"(magic));
  return r;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

}  // namespace tq4
