// Host-side internals shared by the tq4 translation units: the weight handle, device buffers,
// error reporting.
#pragma once

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>
#include <type_traits>
#include <utility>

#include "common.cuh"

namespace tq4 {

// Thread-local last error message (tq4_last_error).
void set_error(const char* fmt, ...);
void clear_error();

// Switches to `dev` for the duration of a call (RAII).
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    else if (prev == dev) prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

inline int dtype_size(tq4_dtype t) {
  switch (t) {
    case TQ4_F32: return 4;
    case TQ4_F16: return 2;
    case TQ4_BF16: return 2;
    case TQ4_U8: return 1;
  }
  return 0;
}

inline const char* dtype_name(tq4_dtype t) {
  switch (t) {
    case TQ4_F32: return "f32";
    case TQ4_F16: return "f16";
    case TQ4_BF16: return "bf16";
    case TQ4_U8: return "u8";
  }
  return "?";
}

#define TQ4_TRY(expr)                      \
  do {                                     \
    tq4_status _s = (expr);                \
    if (_s != TQ4_OK) return _s;           \
  } while (0)

#define TQ4_CUDA(expr)                                                                      \
  do {                                                                                      \
    cudaError_t _e = (expr);                                                                \
    if (_e != cudaSuccess) {                                                                \
      ::tq4::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__,    \
                       __LINE__);                                                           \
      return _e == cudaErrorMemoryAllocation ? TQ4_ERR_OUT_OF_MEMORY : TQ4_ERR_CUDA;        \
    }                                                                                       \
  } while (0)

// Launch with the programmatic-stream-serialization attribute (see pdl_wait in common.cuh), unless
// the environment sets TQ4_PDL=0, in which case it is an ordinary launch.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) applies to the device that is current when it
// is called, so it is made once per (kernel, device): `done` holds one bit per device (ordinals
// 0..63). Two threads may both set it the first time; the call is idempotent.
template <typename F>
cudaError_t set_smem_limit_once(F kern, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool tracked = dev >= 0 && dev < 64;
  if (tracked && ((done.load(std::memory_order_acquire) >> dev) & 1u)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && tracked) done.fetch_or(uint64_t(1) << dev, std::memory_order_acq_rel);
  return e;
}

// A device allocation owned by a handle (freed on destruction).
struct DeviceBuffer {
  void* ptr = nullptr;
  int64_t bytes = 0;
  DeviceBuffer() = default;
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  ~DeviceBuffer() { release(); }
  tq4_status alloc(int64_t n) {
    release();
    if (n <= 0) return TQ4_OK;
    cudaError_t e = cudaMalloc(&ptr, (size_t)n);
    if (e != cudaSuccess) {
      ptr = nullptr;
      set_error("cudaMalloc(%lld bytes) failed: %s", (long long)n, cudaGetErrorString(e));
      return e == cudaErrorMemoryAllocation ? TQ4_ERR_OUT_OF_MEMORY : TQ4_ERR_CUDA;
    }
    bytes = n;
    return TQ4_OK;
  }
  void release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
  }
};

}  // namespace tq4

// The weight handle: the node's attributes and its device buffers in the handle's layout.
struct tq4_weight {
  tq4_weight_desc desc{};
  int device = 0;
  int64_t blocks = 0;      // ceil(K / block_size)
  int64_t k_pad = 0;       // K rounded up to whole 64-byte groups
  int64_t row_bytes = 0;   // k_pad * bits / 8, a multiple of 64
  int64_t groups = 0;      // row_bytes / 64
  int64_t n_pad = 0;       // N rounded up to 128 rows
  int64_t blocks_pad = 0;  // blocks per row of the scale / zero-point arrays
  int bs_log2 = 0;
  float z_const = 0.f;     // 2^(bits-1) when the node has no zero points
  cudaStream_t stream = nullptr;  // the handle's own stream (creation work only)
  tq4::DeviceBuffer q;       // [n_pad][row_bytes]
  tq4::DeviceBuffer scales;  // [blocks_pad][n_pad] in T (block-major)
  tq4::DeviceBuffer zps;     // [blocks_pad][n_pad] in T, or empty
  // [n_pad] int32, T = f32 with 4-bit weights only: |(q - z) * s| <= 2^wexp[n] over row n. The
  // tensor-core GEMM carries row n's weights as f16 (q - z) * s * 2^-wexp[n] (kept in the normal
  // f16 range) and multiplies its outputs back by 2^wexp[n].
  tq4::DeviceBuffer wexp;
  // [blocks_pad][n_pad] f16, f32 4-bit weights without zero points: RN_f16(s * 2^-wexp[n]), the
  // tensor-core GEMM's block scales (read by TMA like 2-byte scales; one rounding more than
  // scaling the f32 product). Empty otherwise.
  tq4::DeviceBuffer scales16;
  int num_sms = 148;
  // split-K workspaces of the GEMV, one per CUDA stream (a tq4::WorkspaceMap, made on first use)
  void* ws_mutex = nullptr;
  // TMA descriptors for the GEMM's tile widths (128, 96, 64), made at creation: packed rows,
  // block-major scales and zero points
  alignas(64) CUtensorMap wmaps[3];
  alignas(64) CUtensorMap smaps[3];
  alignas(64) CUtensorMap zmaps[3];
  bool wmaps_ok = false;
  alignas(64) CUtensorMap smap16;  // scales16 with the GEMM's box, when scales16 exists
  bool s16_ok = false;
  // TMA descriptors of the GEMV: 128 packed rows x 64 bytes, and 136 rows x gv_nbs blocks of the
  // scales / zero points; gv_gps groups per pipeline stage
  alignas(64) CUtensorMap gv_wmap;
  alignas(64) CUtensorMap gv_smap;
  alignas(64) CUtensorMap gv_zmap;
  bool gv_maps_ok = false;
  int gv_gps = 1, gv_nbs = 1;
  // TMA descriptors of the 32-row-unit M = 1 GEMV (4-bit weights of at most 8 packed groups per
  // row): 32 packed rows x 64 bytes, and 40 rows x all blocks of the scales / zero points
  alignas(64) CUtensorMap rw_wmap;
  alignas(64) CUtensorMap rw_smap;
  alignas(64) CUtensorMap rw_zmap;
  bool rw_ok = false;
};

namespace tq4 {
using Weight = tq4_weight;

// Where one raw input of a weight comes from: `length` bytes of memory at `data` (host or device),
// or, when `path` is set, `length` bytes of that file from `offset` (ONNX external data).
struct Source {
  const void* data = nullptr;
  std::string path;
  int64_t offset = 0;
  int64_t length = 0;
};
// Checks one tq4_source against the byte count `expect` the descriptor implies, resolving a file
// range that runs to the end of the file; `what` names the input in the message.
tq4_status resolve_source(const tq4_source* in, int64_t expect, const char* what, Source* out);
// Copies a source's bytes to `dst` (device memory of `device`, the current device). Memory copies
// are queued on `st`; a file range is read by host threads and has reached the device on return.
tq4_status fill_device(void* dst, const Source& src, int device, cudaStream_t st);
// Stages the raw inputs on the device and rewrites them into the handle's layout; `zp` is null
// when the weight has no zero-point input.
tq4_status prepare_weight(Weight& w, const Source& b, const Source& scales, const Source* zp);
// Fills a handle laid out for the summed N with the rows of `parts` in order (tq4_weight_merge).
tq4_status merge_weight(Weight& w, const Weight* const* parts, int count);
tq4_status make_weight_maps(Weight& w);
tq4_status make_gemv_maps(Weight& w);
// A 2-D tiled TMA descriptor (cuTensorMapEncodeTiled through the runtime's driver entry point).
tq4_status make_map(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t inner,
                    uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle sw);
tq4_status run_dequant(const Weight& w, const int64_t* rows, int64_t n_out, void* out, cudaStream_t st);
// Y rows have a stride of `ldy` elements (N for a dense Y; the shard width for a sharded call).
tq4_status run_gemv(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                    tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st);
tq4_status run_gemm(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                    tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st);
tq4_status run_matmul(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                      tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st);
}  // namespace tq4
