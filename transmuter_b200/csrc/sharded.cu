// N-sharded MatMulNBits: each rank holds rows [first, first+count) of B, scales and zero points,
// computes its columns of Y, and Y is assembled on every rank over NVLink. The reference has no
// device collective; this serves the very wide projections (the 151936-column lm_head) named by
// the north star.
//
// Assembly of large outputs (a slice of 4 MB or more): each rank computes its slice into a
// buffer that every peer has mapped (CUDA IPC handles, exchanged once through NCCL). One exchange
// kernel then, with e this call's epoch (a device counter, so graph replays advance it): (1)
// stores e into every rank's "ready" flags (release, system scope); (2) waits, bounded, until all
// ranks' ready flags carry e; (3) loads every rank's slice over NVLink straight into Y's [M][N]
// layout; (4) in its last block stores e into every rank's "read" flags and waits until every
// rank has read this rank's slice, so the next call's compute never overwrites a slice that a
// peer is still reading. Small outputs, where NCCL's latency measured lower, and hosts where
// peer mapping is not available on every rank use NCCL's all-gather (plus a reordering kernel
// for M > 1).
//
// NCCL is loaded with dlopen at first use, so the library loads on hosts without NCCL and links
// to whichever libnccl.so.2 the process already has (torch's, when torch is imported first).
// Communicators are non-blocking: initialisation polls ncclCommGetAsyncError against a host
// deadline and aborts the communicator when the deadline passes.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "internal.cuh"
#include "rows.cuh"

namespace tq4 {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi* nccl_api() {
  static NcclApi api;
  static bool tried = false;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (tried) return api.handle ? &api : nullptr;
  tried = true;
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char* n : names) {
    api.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (api.handle) break;
  }
  if (!api.handle) return nullptr;
#define TQ4_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(api.handle, name))
  TQ4_SYM(GetUniqueId, "ncclGetUniqueId");
  TQ4_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
  TQ4_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
  TQ4_SYM(CommAbort, "ncclCommAbort");
  TQ4_SYM(CommDestroy, "ncclCommDestroy");
  TQ4_SYM(AllGather, "ncclAllGather");
  TQ4_SYM(GetErrorString, "ncclGetErrorString");
#undef TQ4_SYM
  if (!api.GetUniqueId || !api.CommInitRankConfig || !api.CommGetAsyncError || !api.CommAbort ||
      !api.CommDestroy || !api.AllGather || !api.GetErrorString) {
    dlclose(api.handle);
    api.handle = nullptr;
    return nullptr;
  }
  return &api;
}

static tq4_status need_nccl(NcclApi** out) {
  *out = nccl_api();
  if (!*out) {
    set_error("NCCL is not available (dlopen libnccl.so.2 failed or lacks symbols)");
    return TQ4_ERR_NCCL;
  }
  return TQ4_OK;
}

// Waits until a non-blocking communicator leaves ncclInProgress, at most until `deadline`.
static tq4_status nccl_wait(NcclApi* api, ncclComm_t comm,
                            std::chrono::steady_clock::time_point deadline, const char* what) {
  for (;;) {
    ncclResult_t state = ncclSuccess;
    ncclResult_t r = api->CommGetAsyncError(comm, &state);
    if (r != ncclSuccess) state = r;
    if (state == ncclSuccess) return TQ4_OK;
    if (state != ncclInProgress) {
      set_error("%s: %s", what, api->GetErrorString(state));
      return TQ4_ERR_NCCL;
    }
    if (std::chrono::steady_clock::now() > deadline) {
      set_error("%s: timed out waiting for the other ranks", what);
      return TQ4_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

static ncclDataType_t nccl_type(tq4_dtype t) {
  switch (t) {
    case TQ4_F16: return ncclFloat16;
    case TQ4_BF16: return ncclBfloat16;
    default: return ncclFloat32;
  }
}

constexpr int kMaxPeers = 8;

// Flag words of a rank: ready[kMaxPeers], read[kMaxPeers], then the block counter and the epoch.
constexpr int kFlagReady = 0, kFlagRead = kMaxPeers, kFlagCounter = 2 * kMaxPeers, kFlagEpoch = 2 * kMaxPeers + 1;
constexpr int kFlagWords = 2 * kMaxPeers + 2;
constexpr int64_t kPeerMinSlice = 4 << 20;  // bytes per rank below which NCCL assembles Y

struct PeerArgs {
  const uint8_t* slice[kMaxPeers];       // rank q's [M][share] slice (own or peer-mapped)
  unsigned long long* flags[kMaxPeers];  // rank q's flag words (own or peer-mapped)
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until flags[base + q] >= epoch for every rank q other than `skip`; false (and the
// device status) on timeout.
__device__ __forceinline__ bool wait_flags(const unsigned long long* flags, int base, int nranks,
                                           unsigned long long epoch, int skip = -1) {
  const long long t0 = clock64(), limit = wait_limit();
  for (int q = 0; q < nranks; ++q) {
    if (q == skip) continue;
    while (ld_acquire_sys(flags + base + q) < epoch) {
      if (clock64() - t0 > limit) {
        report(kDevTimeoutPeer);
        return false;
      }
    }
  }
  return true;
}

// Publish this rank's slice, wait for every rank's, gather Y [M][N] (16-byte chunks where
// aligned); see the top of this file.
constexpr int kExThreads = 256;

// See the top of this file.
__global__ void __launch_bounds__(kExThreads) exchange_kernel(PeerArgs pa, unsigned long long* own, int rank,
                                                              int nranks, int64_t m, int64_t share, int64_t n, int ys,
                                                              uint8_t* y) {
  __shared__ int s_ok;
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long*>(own + kFlagEpoch) + 1;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      __threadfence_system();  // the slice (written by the previous kernel) before the flag
      for (int q = 0; q < nranks; ++q) st_release_sys(pa.flags[q] + kFlagReady + rank, epoch);
    }
    s_ok = wait_flags(own, kFlagReady, nranks, epoch);
  }
  __syncthreads();
  if (s_ok) {
    const int64_t row_bytes = share * ys;       // a multiple of 32
    const int64_t chunks_row = row_bytes / 16;  // per slice row
    const int64_t total = m * nranks * chunks_row;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t c = i % chunks_row, rq = i / chunks_row;
      const int q = (int)(rq % nranks);
      const int64_t row = rq / nranks;
      const int64_t col0 = q * share + c * (16 / ys);  // first Y column of the chunk
      if (col0 >= n) continue;
      const uint8_t* src = pa.slice[q] + row * row_bytes + c * 16;
      uint8_t* dst = y + (row * n + col0) * ys;
      if (col0 + 16 / ys <= n && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
      } else {
        for (int e = 0; e < 16 / ys && col0 + e < n; ++e)
          for (int b = 0; b < ys; ++b) dst[e * ys + b] = src[e * ys + b];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int* counter = reinterpret_cast<unsigned int*>(own + kFlagCounter);
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {  // the last block: this rank read every slice
      *counter = 0;
      __threadfence_system();
      for (int q = 0; q < nranks; ++q) st_release_sys(pa.flags[q] + kFlagRead + rank, epoch);
      wait_flags(own, kFlagRead, nranks, epoch);  // every rank has read this rank's slice
      *reinterpret_cast<volatile unsigned long long*>(own + kFlagEpoch) = epoch;
    }
  }
}

// The assembly of an N-sharded M = 1 call (the push path). Every rank's GEMV (gemv_rows.cu) has
// stored its columns into half (e & 1) of every rank's assembly buffer over NVLink, e being this
// call's epoch. Block 0 publishes e in every peer's ready flags (a relaxed system-scope store once
// the GEMV, the previous grid, has completed); every block waits, bounded, for every
// peer's flag, then copies its share of the assembled row into Y; the last block to finish
// advances the epoch. Two halves suffice: a rank's GEMV of call e + 1 runs only after its own
// assembly of call e, which saw every peer's flag e, set by each peer after its assembly of
// call e - 1, the last reader of the half that call e + 1 writes.
__global__ void __launch_bounds__(kExThreads) push_finish_kernel(PeerArgs pa, unsigned long long* own, int rank,
                                                                 int nranks, const uint8_t* assembly,
                                                                 int64_t half_bytes, uint8_t* y, int64_t y_bytes) {
  __shared__ int s_ok;
  // Launched with programmatic dependent launch: once pdl_wait() returns, the GEMV before it has
  // completed and its memory operations are performed, its stores into the peers' assembly
  // buffers included (griddepcontrol.wait). Only then may the next call's GEMV start, and its
  // weight loads (all it does before its own pdl_wait) overlap this kernel's wait for the peers
  // and its copy.
  pdl_wait();
  pdl_trigger();
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long*>(own + kFlagEpoch) + 1;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      // The data this flag announces was written by the previous grid, whose stores are already
      // performed at the peers (above), so the flag needs no release: a system-scope fence or a
      // st.release.sys here cost about 2 us each (globaltimer stamps on two B200s: 5.4 us from
      // this point until the peer's flag was seen with both, 1.7 us with the relaxed store).
      for (int q = 0; q < nranks; ++q)
        if (q != rank) st_relaxed_sys(pa.flags[q] + kFlagReady + rank, epoch);
    }
    s_ok = wait_flags(own, kFlagReady, nranks, epoch, rank);
  }
  __syncthreads();
  if (s_ok) {
    const uint8_t* src = assembly + (int64_t)(epoch & 1) * half_bytes;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t head = 0;
    if (((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(src)) & 15) == 0) {
      const int64_t n16 = y_bytes / 16;
      for (int64_t i = tid; i < n16; i += stride)
        reinterpret_cast<uint4*>(y)[i] = __ldcg(reinterpret_cast<const uint4*>(src) + i);
      head = n16 * 16;
    }
    for (int64_t i = head + tid; i < y_bytes; i += stride) y[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int* counter = reinterpret_cast<unsigned int*>(own + kFlagCounter);
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {  // the last block: the call is over
      *counter = 0;
      *reinterpret_cast<volatile unsigned long long*>(own + kFlagEpoch) = epoch;
    }
  }
}

// The peer-flag wait of the kernels above on a flag that nothing sets (tq4_selftest_peer_wait):
// it runs out after the device's wait limit and reports kDevTimeoutPeer.
__device__ unsigned long long g_never_set[kMaxPeers];
__global__ void selftest_peer_wait_kernel() {
  if (threadIdx.x == 0) wait_flags(g_never_set, 0, 2, 1);
}

// [P][M][share] (the all-gather order) -> Y [M][N]
template <typename T>
__global__ void unshard_kernel(const T* __restrict__ g, int64_t m, int64_t share, int nranks,
                               int64_t n, T* __restrict__ y) {
  const int64_t total = m * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / n, col = i % n;
    const int64_t r = col / share, j = col % share;
    y[i] = g[(r * m + row) * share + j];
  }
}

}  // namespace tq4

using namespace tq4;

struct tq4_comm {
  ncclComm_t comm = nullptr;
  int nranks = 1, rank = 0, device = 0;
  bool broken = false;
};

struct tq4_sharded {
  tq4_comm* comm = nullptr;
  tq4_weight* local = nullptr;  // null when this rank owns no rows
  tq4_weight_desc desc{};       // the full weight
  int64_t share = 0;            // rows per rank (a multiple of 16), the all-gather unit
  int64_t first = 0, count = 0;
  std::mutex mu;
  DeviceBuffer part;    // this rank's [M][share] output (NCCL path)
  DeviceBuffer gather;  // [P][M][share] (NCCL path)
  // Peer memory (CUDA IPC mappings; each set is mapped on every rank or on none).
  // The flag words of every rank (ready, read, block counter, epoch):
  bool flags_tried = false, flags_ok = false;
  DeviceBuffer flags;
  void* peer_flags[kMaxPeers] = {};
  // The exchange's [M][share] slices:
  bool slice_tried = false, slice_ok = false;
  int64_t slice_cap = 0;
  DeviceBuffer slice;
  void* peer_slice[kMaxPeers] = {};
  // The M = 1 push path's assembly buffers (two halves of N outputs, 4 bytes each at most):
  bool asm_tried = false, asm_ok = false;
  DeviceBuffer assembly;
  void* peer_asm[kMaxPeers] = {};
};

namespace tq4 {

tq4_status gemv_workspace(const Weight& w, cudaStream_t st, int64_t ws_bytes, int64_t ctr_count, float** ws,
                          int** counters);

static void close_set(tq4_sharded* s, void** mapped, bool* ok) {
  for (int q = 0; q < s->comm->nranks && q < kMaxPeers; ++q)
    if (q != s->comm->rank && mapped[q]) cudaIpcCloseMemHandle(mapped[q]);
  for (int q = 0; q < kMaxPeers; ++q) mapped[q] = nullptr;
  *ok = false;
}

static tq4_status allgather_bytes(tq4_sharded* s, NcclApi* api, const void* mine, void* all, size_t bytes,
                                  cudaStream_t st) {
  const int P = s->comm->nranks;
  DeviceBuffer buf;
  TQ4_TRY(buf.alloc((int64_t)(P + 1) * bytes));
  uint8_t* d = static_cast<uint8_t*>(buf.ptr);
  TQ4_CUDA(cudaMemcpy(d + P * bytes, mine, bytes, cudaMemcpyHostToDevice));
  ncclResult_t r = api->AllGather(d + P * bytes, d, bytes, ncclUint8, s->comm->comm, st);
  if (r == ncclInProgress) {
    TQ4_TRY(nccl_wait(api, s->comm->comm, std::chrono::steady_clock::now() + std::chrono::seconds(60), "ncclAllGather"));
  } else if (r != ncclSuccess) {
    s->comm->broken = true;
    set_error("ncclAllGather: %s", api->GetErrorString(r));
    return TQ4_ERR_NCCL;
  }
  TQ4_CUDA(cudaStreamSynchronize(st));
  TQ4_CUDA(cudaMemcpy(all, d, P * bytes, cudaMemcpyDeviceToHost));
  return TQ4_OK;
}

// Collective (every rank, same call, outside stream capture): the IPC handle of `local` on every
// rank, each peer's buffer mapped into mapped[] (the own entry is `local`). *ok is set only when
// every rank mapped every peer; otherwise nothing stays mapped.
static tq4_status map_set(tq4_sharded* s, NcclApi* api, void* local, void** mapped, bool* ok, cudaStream_t st) {
  const int P = s->comm->nranks, R = s->comm->rank;
  *ok = false;
  cudaIpcMemHandle_t mine{};
  bool good = cudaIpcGetMemHandle(&mine, local) == cudaSuccess;
  cudaGetLastError();
  cudaIpcMemHandle_t all[kMaxPeers];
  TQ4_TRY(allgather_bytes(s, api, &mine, all, sizeof(mine), st));
  for (int q = 0; q < P; ++q) {
    if (q == R) {
      mapped[q] = local;
      continue;
    }
    void* ptr = nullptr;
    if (!good || cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      good = false;
      continue;
    }
    mapped[q] = ptr;
  }
  const uint8_t mine_ok = good ? 1 : 0;
  uint8_t oks[kMaxPeers];
  TQ4_TRY(allgather_bytes(s, api, &mine_ok, oks, 1, st));
  bool all_ok = true;
  for (int q = 0; q < P; ++q) all_ok = all_ok && oks[q];
  if (!all_ok) {
    close_set(s, mapped, ok);
    return TQ4_OK;
  }
  *ok = true;
  return TQ4_OK;
}

static tq4_status not_capturing(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  TQ4_CUDA(cudaStreamIsCapturing(st, &cs));
  if (cs != cudaStreamCaptureStatusNone) {
    set_error("tq4_sharded_matmul: the first call of a new shape must come before stream capture");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  return TQ4_OK;
}

// Collective: every rank's flag words mapped (once; the epochs only grow, so they outlive any
// regrowth of the data buffers).
static tq4_status ensure_flags(tq4_sharded* s, NcclApi* api, cudaStream_t st) {
  if (s->flags_tried) return TQ4_OK;
  if (s->comm->nranks > kMaxPeers) {
    s->flags_tried = true;
    return TQ4_OK;
  }
  TQ4_TRY(not_capturing(st));
  TQ4_CUDA(cudaStreamSynchronize(st));
  s->flags_tried = true;
  TQ4_TRY(s->flags.alloc(kFlagWords * sizeof(unsigned long long)));
  TQ4_CUDA(cudaMemset(s->flags.ptr, 0, kFlagWords * sizeof(unsigned long long)));
  return map_set(s, api, s->flags.ptr, s->peer_flags, &s->flags_ok, st);
}

// Collective: slice buffers of at least `bytes` on every rank, mapped by every peer.
static tq4_status ensure_slices(tq4_sharded* s, NcclApi* api, int64_t bytes, cudaStream_t st) {
  TQ4_TRY(ensure_flags(s, api, st));
  if (!s->flags_ok) return TQ4_OK;
  if (s->slice_tried && (!s->slice_ok || s->slice_cap >= bytes)) return TQ4_OK;
  TQ4_TRY(not_capturing(st));
  TQ4_CUDA(cudaStreamSynchronize(st));
  if (s->slice_tried) {  // growing: every rank is here too (the same collective call)
    close_set(s, s->peer_slice, &s->slice_ok);
    TQ4_CUDA(cudaDeviceSynchronize());
  }
  s->slice_tried = true;
  const int64_t cap = (bytes + (2 << 20) - 1) / (2 << 20) * (2 << 20);
  TQ4_TRY(s->slice.alloc(cap));
  TQ4_TRY(map_set(s, api, s->slice.ptr, s->peer_slice, &s->slice_ok, st));
  if (s->slice_ok) s->slice_cap = cap;
  return TQ4_OK;
}

// Elements of one half of an assembly buffer: N rounded up to 16, so that the second half starts
// 16-byte aligned for 2- and 4-byte outputs (push_finish_kernel copies it in 16-byte words).
static int64_t assembly_half_elems(const tq4_sharded* s) { return (s->desc.N + 15) / 16 * 16; }

// Collective: the M = 1 assembly buffers (2 halves of N outputs of up to 4 bytes), mapped by every
// peer.
static tq4_status ensure_assembly(tq4_sharded* s, NcclApi* api, cudaStream_t st) {
  TQ4_TRY(ensure_flags(s, api, st));
  if (!s->flags_ok || s->asm_tried) return TQ4_OK;
  TQ4_TRY(not_capturing(st));
  TQ4_CUDA(cudaStreamSynchronize(st));
  s->asm_tried = true;
  TQ4_TRY(s->assembly.alloc(2 * assembly_half_elems(s) * 4));
  return map_set(s, api, s->assembly.ptr, s->peer_asm, &s->asm_ok, st);
}

// Whether an N-sharded M = 1 call takes the push path: the 32-row-unit GEMV takes every rank's
// rows (4-bit weights of at most 8 packed groups per row; a property of the full weight, so every
// rank decides alike) and there are at most 8 ranks.
static bool push_shape(const tq4_sharded* s, int64_t m) {
  const tq4_weight_desc& d = s->desc;
  const int64_t blocks = (d.K + d.block_size - 1) / d.block_size;
  const int64_t groups = (blocks * d.block_size * d.bits / 8 + 63) / 64;
  return m == 1 && d.bits == 4 && groups <= 8 && s->comm->nranks > 1 && s->comm->nranks <= kMaxPeers;
}

}  // namespace tq4

extern "C" {

tq4_status tq4_comm_unique_id(unsigned char id[TQ4_UNIQUE_ID_BYTES]) {
  NcclApi* api;
  TQ4_TRY(need_nccl(&api));
  if (!id) {
    set_error("tq4_comm_unique_id: null output");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  ncclUniqueId uid;
  ncclResult_t r = api->GetUniqueId(&uid);
  if (r != ncclSuccess) {
    set_error("ncclGetUniqueId: %s", api->GetErrorString(r));
    return TQ4_ERR_NCCL;
  }
  static_assert(sizeof(uid.internal) == TQ4_UNIQUE_ID_BYTES, "NCCL unique id size");
  memcpy(id, uid.internal, TQ4_UNIQUE_ID_BYTES);
  return TQ4_OK;
}

tq4_status tq4_comm_create(const unsigned char id[TQ4_UNIQUE_ID_BYTES], int nranks, int rank,
                           int device, int timeout_ms, tq4_comm** out) {
  if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks) {
    set_error("tq4_comm_create: bad arguments (nranks=%d, rank=%d)", nranks, rank);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  *out = nullptr;
  NcclApi* api;
  TQ4_TRY(need_nccl(&api));
  TQ4_CUDA(cudaSetDevice(device));
  ncclUniqueId uid;
  memcpy(uid.internal, id, TQ4_UNIQUE_ID_BYTES);
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  tq4_comm* c = new tq4_comm();
  c->nranks = nranks;
  c->rank = rank;
  c->device = device;
  ncclResult_t r = api->CommInitRankConfig(&c->comm, nranks, uid, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) {
    set_error("ncclCommInitRankConfig: %s", api->GetErrorString(r));
    delete c;
    return TQ4_ERR_NCCL;
  }
  const auto deadline = std::chrono::steady_clock::now() +
                        std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 60000);
  tq4_status st = nccl_wait(api, c->comm, deadline, "ncclCommInitRankConfig");
  if (st != TQ4_OK) {
    api->CommAbort(c->comm);
    delete c;
    return st;
  }
  *out = c;
  return TQ4_OK;
}

tq4_status tq4_comm_destroy(tq4_comm* c) {
  if (!c) return TQ4_OK;
  NcclApi* api = nccl_api();
  if (api && c->comm) {
    ncclResult_t state = ncclSuccess;
    api->CommGetAsyncError(c->comm, &state);
    if (c->broken || (state != ncclSuccess && state != ncclInProgress)) api->CommAbort(c->comm);
    else api->CommDestroy(c->comm);
  }
  delete c;
  return TQ4_OK;
}

// A sharded handle without its local weight: this rank's share of the N rows.
static tq4_sharded* new_sharded(const tq4_weight_desc* d, tq4_comm* comm) {
  tq4_sharded* s = new tq4_sharded();
  s->comm = comm;
  s->desc = *d;
  const int64_t P = comm->nranks;
  s->share = ((d->N + P - 1) / P + 15) / 16 * 16;
  s->first = std::min<int64_t>(d->N, comm->rank * s->share);
  s->count = std::min<int64_t>(d->N - s->first, s->share);
  return s;
}

tq4_status tq4_sharded_create(const tq4_weight_desc* d, const void* b, int64_t b_bytes,
                              const void* scales, const void* zp, tq4_comm* comm,
                              tq4_sharded** out) {
  if (!out || !comm || !d) {
    set_error("tq4_sharded_create: null argument");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  *out = nullptr;
  int64_t need_b = 0;
  TQ4_TRY(tq4_weight_input_sizes(d, &need_b, nullptr, nullptr));
  if (b_bytes != need_b || !b || !scales || (d->zp_kind != TQ4_ZP_NONE && !zp)) {
    set_error("tq4_sharded_create: B has %lld bytes (expected %lld) or an input is missing",
              (long long)b_bytes, (long long)need_b);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  tq4_sharded* s = new_sharded(d, comm);
  if (s->count > 0) {
    const int64_t blocks = (d->K + d->block_size - 1) / d->block_size;
    const int64_t raw_row = blocks * d->block_size * d->bits / 8;
    tq4_weight_desc ld = *d;
    ld.N = s->count;
    const uint8_t* bb = static_cast<const uint8_t*>(b) + s->first * raw_row;
    const uint8_t* sb = static_cast<const uint8_t*>(scales) + s->first * blocks * dtype_size(d->scale_dtype);
    const uint8_t* zb = nullptr;
    if (d->zp_kind == TQ4_ZP_PACKED) zb = static_cast<const uint8_t*>(zp) + s->first * ((blocks * d->bits + 7) / 8);
    if (d->zp_kind == TQ4_ZP_FLOAT) zb = static_cast<const uint8_t*>(zp) + s->first * blocks * dtype_size(d->zp_dtype);
    tq4_status st = tq4_weight_create(&ld, bb, s->count * raw_row, sb, zb, comm->device, &s->local);
    if (st != TQ4_OK) {
      delete s;
      return st;
    }
  }
  *out = s;
  return TQ4_OK;
}

tq4_status tq4_sharded_create_from(const tq4_weight_desc* d, const tq4_source* b,
                                   const tq4_source* scales, const tq4_source* zp, tq4_comm* comm,
                                   tq4_sharded** out) {
  if (!out || !comm || !d) {
    set_error("tq4_sharded_create_from: null argument");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  *out = nullptr;
  int64_t b_bytes = 0, s_bytes = 0, z_bytes = 0;
  TQ4_TRY(tq4_weight_input_sizes(d, &b_bytes, &s_bytes, &z_bytes));
  // The full inputs are checked (files, ranges, sizes) on every rank before any device work.
  Source fb, fs, fz;
  TQ4_TRY(resolve_source(b, b_bytes, "B", &fb));
  TQ4_TRY(resolve_source(scales, s_bytes, "scales", &fs));
  const bool has_zp = d->zp_kind != TQ4_ZP_NONE;
  if (has_zp) {
    if (!zp) {
      set_error("MatMulNBits: zero points declared but not given");
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    TQ4_TRY(resolve_source(zp, z_bytes, "zero points", &fz));
  }
  tq4_sharded* s = new_sharded(d, comm);
  if (s->count > 0) {
    // Every input is N rows of equal size, so this rank's rows are one contiguous range of each:
    // a file range is narrowed, and the rank reads only its rows.
    auto rows_of = [&](const Source& src, int64_t total) {
      const int64_t row = total / d->N;
      tq4_source t{};
      if (src.path.empty()) {
        t.data = static_cast<const uint8_t*>(src.data) + s->first * row;
      } else {
        t.path = src.path.c_str();
        t.offset = src.offset + s->first * row;
      }
      t.length = s->count * row;
      return t;
    };
    tq4_weight_desc ld = *d;
    ld.N = s->count;
    const tq4_source lb = rows_of(fb, b_bytes), ls = rows_of(fs, s_bytes);
    const tq4_source lz = has_zp ? rows_of(fz, z_bytes) : tq4_source{};
    const tq4_status st = tq4_weight_create_from(&ld, &lb, &ls, has_zp ? &lz : nullptr, comm->device, &s->local);
    if (st != TQ4_OK) {
      delete s;
      return st;
    }
  }
  *out = s;
  return TQ4_OK;
}

tq4_status tq4_sharded_rows(const tq4_sharded* s, int64_t* first, int64_t* count) {
  if (!s) {
    set_error("tq4_sharded_rows: null handle");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (first) *first = s->first;
  if (count) *count = s->count;
  return TQ4_OK;
}

tq4_status tq4_sharded_matmul(const tq4_sharded* cs, const void* a, int64_t m, tq4_dtype a_t,
                              const void* bias, tq4_dtype bias_t, void* y, tq4_dtype y_t,
                              void* stream) {
  tq4_sharded* s = const_cast<tq4_sharded*>(cs);
  if (!s || m < 0 || (m > 0 && (!a || !y))) {
    set_error("tq4_sharded_matmul: bad arguments");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (m == 0) return TQ4_OK;
  NcclApi* api;
  TQ4_TRY(need_nccl(&api));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t P = s->comm->nranks;
  const int ys = dtype_size(y_t);
  std::lock_guard<std::mutex> lock(s->mu);
  TQ4_CUDA(cudaSetDevice(s->comm->device));
  if (push_shape(s, m)) {
    // One activation row: every rank's GEMV stores its columns straight into every rank's
    // assembly buffer, then push_finish_kernel exchanges one epoch flag per peer and copies the
    // assembled row into Y.
    TQ4_TRY(ensure_assembly(s, api, st));
    if (s->asm_ok) {
      if (s->local) {
        if (!rows_eligible(*s->local)) {
          set_error("tq4_sharded_matmul: this rank's rows have no 32-row unit descriptors");
          return TQ4_ERR_UNSUPPORTED;
        }
        float* ws = nullptr;
        int* ctr = nullptr;
        TQ4_TRY(gemv_workspace(*s->local, st, 0, 1, &ws, &ctr));
        RowsDst dst;
        for (int q = 0; q < P; ++q) dst.y[q] = s->peer_asm[q];
        dst.ndst = (int)P;
        dst.col0 = s->first;
        dst.epoch = static_cast<const unsigned long long*>(s->flags.ptr) + kFlagEpoch;
        dst.half_elems = assembly_half_elems(s);
        const void* lb = bias ? static_cast<const uint8_t*>(bias) + s->first * dtype_size(bias_t) : nullptr;
        TQ4_TRY(run_gemv_rows(*s->local, a, a_t, lb, bias_t, y_t, dst, ctr, st));
      }
      PeerArgs pa{};
      for (int q = 0; q < P; ++q) pa.flags[q] = static_cast<unsigned long long*>(s->peer_flags[q]);
      const int64_t y_bytes = s->desc.N * ys;
      const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((y_bytes / 16 + kExThreads - 1) / kExThreads, 148));
      TQ4_CUDA(launch_pdl(push_finish_kernel, dim3(grid), dim3(kExThreads), 0, st, pa,
                          static_cast<unsigned long long*>(s->flags.ptr), s->comm->rank, (int)P,
                          static_cast<const uint8_t*>(s->assembly.ptr), assembly_half_elems(s) * ys,
                          static_cast<uint8_t*>(y), y_bytes));
      return TQ4_OK;
    }
  }
  const bool large = m * s->share * ys >= kPeerMinSlice;
  if (large) TQ4_TRY(ensure_slices(s, api, m * s->share * ys, st));
  if (large && s->slice_ok) {
    if (s->local) {
      const void* lb = bias ? static_cast<const uint8_t*>(bias) + s->first * dtype_size(bias_t) : nullptr;
      TQ4_TRY(run_matmul(*s->local, a, m, a_t, lb, bias_t, s->slice.ptr, y_t, s->share, st));
    }
    PeerArgs pa{};
    for (int q = 0; q < P; ++q) {
      pa.slice[q] = static_cast<const uint8_t*>(s->peer_slice[q]);
      pa.flags[q] = static_cast<unsigned long long*>(s->peer_flags[q]);
    }
    const int64_t chunks = m * P * (s->share * ys / 16);
    // Every block waits for the last one's signal, so the grid must be resident all at once: no
    // more blocks than the SMs hold together (occupancy of this kernel, looked up once per device).
    static std::atomic<int> resident[64];  // zero-initialised (static storage)
    int dev = s->comm->device;
    if (dev < 0 || dev >= 64) dev = 0;
    int res = resident[dev].load(std::memory_order_relaxed);
    if (res == 0) {
      int per_sm = 0, sms = 0;
      TQ4_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, exchange_kernel, kExThreads, 0));
      TQ4_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, s->comm->device));
      res = std::max(1, per_sm * sms);
      resident[dev].store(res, std::memory_order_relaxed);
    }
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((chunks + kExThreads - 1) / kExThreads,
                                                                  std::min(res, 4 * 148)));
    exchange_kernel<<<grid, kExThreads, 0, st>>>(pa, static_cast<unsigned long long*>(s->flags.ptr), s->comm->rank,
                                                 (int)P, m, s->share, s->desc.N, ys, static_cast<uint8_t*>(y));
    TQ4_CUDA(cudaGetLastError());
    return TQ4_OK;
  }
  // Y itself is the gather target when it already has the [P][1][share] layout.
  const bool direct = (m == 1 && s->share * P == s->desc.N);
  if (s->part.bytes < m * s->share * ys) TQ4_TRY(s->part.alloc(m * s->share * ys));
  if (!direct && s->gather.bytes < P * m * s->share * ys) TQ4_TRY(s->gather.alloc(P * m * s->share * ys));
  if (s->local) {
    const void* lb = bias ? static_cast<const uint8_t*>(bias) + s->first * dtype_size(bias_t) : nullptr;
    TQ4_TRY(run_matmul(*s->local, a, m, a_t, lb, bias_t, s->part.ptr, y_t, s->share, st));
  }
  // rows of a short (or empty) shard beyond `count` are never read back: no clearing needed
  void* dst = direct ? y : s->gather.ptr;
  ncclResult_t r = api->AllGather(s->part.ptr, dst, (size_t)(m * s->share), nccl_type(y_t),
                                  s->comm->comm, st);
  if (r == ncclInProgress) {
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
    TQ4_TRY(nccl_wait(api, s->comm->comm, deadline, "ncclAllGather"));
  } else if (r != ncclSuccess) {
    s->comm->broken = true;
    set_error("ncclAllGather: %s", api->GetErrorString(r));
    return TQ4_ERR_NCCL;
  }
  if (!direct) {
    const int64_t total = m * s->desc.N;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
    switch (y_t) {
      case TQ4_F32:
        unshard_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(s->gather.ptr), m, s->share, (int)P, s->desc.N, static_cast<float*>(y));
        break;
      default:
        unshard_kernel<uint16_t><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(s->gather.ptr), m, s->share, (int)P, s->desc.N, static_cast<uint16_t*>(y));
        break;
    }
    TQ4_CUDA(cudaGetLastError());
  }
  return TQ4_OK;
}

tq4_status tq4_selftest_peer_wait(int device, void* stream) {
  clear_error();
  int ndev = 0;
  TQ4_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) {
    set_error("tq4_selftest_peer_wait: device %d out of range", device);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceGuard guard(device);
  selftest_peer_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  TQ4_CUDA(cudaGetLastError());
  return TQ4_OK;
}

tq4_status tq4_sharded_destroy(tq4_sharded* s) {
  if (!s) return TQ4_OK;
  if (s->local) tq4_weight_destroy(s->local);
  if (s->flags_tried || s->slice_tried || s->asm_tried) {
    cudaSetDevice(s->comm->device);
    cudaDeviceSynchronize();
    close_set(s, s->peer_slice, &s->slice_ok);
    close_set(s, s->peer_asm, &s->asm_ok);
    close_set(s, s->peer_flags, &s->flags_ok);
  }
  s->part.release();
  s->gather.release();
  delete s;
  return TQ4_OK;
}

}  // extern "C"
