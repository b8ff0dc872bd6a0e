// tq4_matmul_noalloc: the decode-shaped MatMulNBits call (M <= 16) for callers that cannot
// allocate device memory.
//
// Who cannot allocate: an Erlang NIF that runs beside EXLA's CUDA client shares the GPU with an
// allocator that reserves most of the device memory up front (EXLA preallocates by default), so
// a cudaMalloc from the NIF can fail at any call; and a caller on a latency-critical decode loop
// cannot afford cudaMalloc / cudaFree, which may synchronize the whole device. tq4_matmul grows a
// per-stream split-K workspace with cudaMalloc on first use; this entry point never allocates.
//
// Its scratch is a file-scope __device__ array of a fixed size. A GPU holds it from the moment
// the library's device code is loaded there until the process exits; under CUDA's default lazy
// module loading that is the first tq4 call on that GPU (any entry point), not the dlopen of the
// library, so a caller that shares the GPU with a preallocating allocator makes one tq4 call per
// GPU before that allocator starts, or runs with CUDA_MODULE_LOADING=EAGER. Host code cannot pass the array's name to a kernel (on
// the host that name is only a stand-in, not a device address), so the first call on each device
// looks up the device address with cudaGetSymbolAddress, with that device current, and keeps it.
// That first call should therefore come before any stream capture. All calls share the one
// array and it keeps the last call's contents: the split-K counters, which must start at zero,
// are cleared by every call that uses them, and calls that overlap on the GPU (different streams,
// or different host threads) race on the scratch.
#include <mutex>

#include "internal.cuh"

namespace tq4 {

// 4 MiB of split-K partial sums and 64 KiB of counters: room for the Llama-3-8B-shaped
// projections at M = 16 (the largest needs 3.5 MiB).
constexpr int64_t kNoAllocScratchFloats = (int64_t)1 << 20;
constexpr int64_t kNoAllocCounters = 16384;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) int g_noalloc_counters[kNoAllocCounters];

struct NoAllocDevice {
  bool ready = false;
  float* scratch = nullptr;
  int* counters = nullptr;
};

constexpr int kMaxDevices = 64;
static NoAllocDevice g_noalloc_devices[kMaxDevices];
static std::mutex g_noalloc_mu;

// Device addresses of the scratch arrays on the current device (looked up once per device).
static tq4_status noalloc_scratch(int device, float** scratch, int** counters) {
  if (device < 0 || device >= kMaxDevices) {
    set_error("tq4_matmul_noalloc: device %d beyond the %d supported", device, kMaxDevices);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_devices[device];
  if (!d.ready) {
    void* s = nullptr;
    void* c = nullptr;
    TQ4_CUDA(cudaGetSymbolAddress(&s, g_noalloc_scratch));
    TQ4_CUDA(cudaGetSymbolAddress(&c, g_noalloc_counters));
    d.scratch = static_cast<float*>(s);
    d.counters = static_cast<int*>(c);
    d.ready = true;
  }
  *scratch = d.scratch;
  *counters = d.counters;
  return TQ4_OK;
}

int64_t gemv_workspace_floats(const Weight& w, int64_t m);
int64_t gemv_counter_count(const Weight& w, int64_t m);
tq4_status run_gemv_with(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                         tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st,
                         float* ws, int* counters, int64_t ws_capacity_floats, int64_t ctr_capacity);

}  // namespace tq4

using namespace tq4;

extern "C" tq4_status tq4_matmul_noalloc(const tq4_weight* w, const void* a, int64_t m,
                                         tq4_dtype a_t, const void* bias, tq4_dtype bias_t,
                                         void* y, tq4_dtype y_t, void* stream) {
  clear_error();
  if (!w) {
    set_error("tq4_matmul_noalloc: null weight handle");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (m < 0) {
    set_error("tq4_matmul_noalloc: M=%lld out of range", (long long)m);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (m > 16) {
    set_error("tq4_matmul_noalloc handles decode-shaped calls (M <= 16); got M=%lld", (long long)m);
    return TQ4_ERR_UNSUPPORTED;
  }
  const bool floats = (a_t == TQ4_F32 || a_t == TQ4_F16 || a_t == TQ4_BF16) &&
                      (y_t == TQ4_F32 || y_t == TQ4_F16 || y_t == TQ4_BF16) &&
                      (!bias || bias_t == TQ4_F32 || bias_t == TQ4_F16 || bias_t == TQ4_BF16);
  if (!floats) {
    set_error("tq4_matmul_noalloc: A, bias and Y must be f32, f16 or bf16");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (m == 0) return TQ4_OK;
  if (!a || !y) {
    set_error("tq4_matmul_noalloc: null A or Y");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  const int64_t need = gemv_workspace_floats(*w, m);
  const int64_t nctr = gemv_counter_count(*w, m);
  if (need > kNoAllocScratchFloats || nctr > kNoAllocCounters) {
    set_error("tq4_matmul_noalloc: this call needs %lld bytes of split-K scratch and %lld counters; "
              "the static limit is %lld bytes and %lld counters (use tq4_matmul)",
              (long long)(need * 4), (long long)nctr, (long long)(kNoAllocScratchFloats * 4),
              (long long)kNoAllocCounters);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceGuard guard(w->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* scratch = nullptr;
  int* counters = nullptr;
  TQ4_TRY(noalloc_scratch(w->device, &scratch, &counters));
  if (nctr > 0) TQ4_CUDA(cudaMemsetAsync(counters, 0, (size_t)nctr * sizeof(int), st));
  return run_gemv_with(*w, a, m, a_t, bias, bias_t, y, y_t, w->desc.N, st, scratch, counters,
                       kNoAllocScratchFloats, kNoAllocCounters);
}
