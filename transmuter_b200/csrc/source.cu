// The raw inputs of a weight handle: memory, or byte ranges of files (ONNX external data).
//
// The reference reads a deferred initializer whole into a binary when the model moves to a
// backend (Transmuter.DeferredTensor.value/1, lib/transmuter/deferred_tensor.ex:27, called by
// move/2 at lib/transmuter.ex:1159; the read itself is Ops.read_external/2,
// lib/transmuter/ops.ex:680-695: "location" joined to the model's directory, "offset" default 0,
// "length" default to the end of the file), and the backend then copies the binary to the device.
// Here the range goes straight to the device: a few reader threads each pread every n-th chunk
// of the range into one of two pinned buffers, and each chunk's host-to-device copy (on the
// thread's own stream) overlaps that thread's next read. The tensor is never whole in host
// memory. The pinned buffers (kMaxReaders x 2 x kChunkBytes = 64 MiB) are allocated by the first
// read of the process and kept for the later ones, since pinning that much memory costs about as
// much as reading a gigabyte from the page cache; reads take turns on them.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <mutex>
#include <thread>
#include <vector>

#include "internal.cuh"

namespace tq4 {

namespace {

constexpr int64_t kChunkBytes = 4ll << 20;
constexpr int kMaxReaders = 8;

// The pinned staging of all file reads: two chunks per reader, portable across devices. Never
// freed: it lives as long as the process (freeing it at exit could run after the CUDA runtime's
// own teardown).
struct Staging {
  std::mutex mu;
  void* slot[kMaxReaders][2] = {};
};

Staging& staging() {
  static Staging* s = new Staging();
  return *s;
}

struct ReadError {
  tq4_status code = TQ4_OK;
  std::string msg;
};

std::string cuda_message(const char* what, cudaError_t e) {
  return std::string(what) + " failed: " + cudaGetErrorString(e);
}

// Reader t of n: chunks t, t + n, t + 2n, ... of the range, into dst (device memory).
void read_chunks(int fd, const Source* src, char* dst, int device, int t, int n, int64_t chunks,
                 void* const* slot, std::atomic<bool>* failed, ReadError* err) {
  auto fail = [&](tq4_status code, std::string msg) {
    if (err->code == TQ4_OK) {
      err->code = code;
      err->msg = std::move(msg);
    }
    failed->store(true);
  };
  cudaError_t ce = cudaSetDevice(device);
  if (ce != cudaSuccess) return fail(TQ4_ERR_CUDA, cuda_message("cudaSetDevice", ce));
  cudaStream_t stream = nullptr;
  cudaEvent_t copied[2] = {nullptr, nullptr};
  bool pending[2] = {false, false};
  ce = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
  if (ce != cudaSuccess) stream = nullptr;
  for (int k = 0; k < 2 && ce == cudaSuccess; ++k)
    ce = cudaEventCreateWithFlags(&copied[k], cudaEventDisableTiming);
  if (ce != cudaSuccess) fail(TQ4_ERR_CUDA, cuda_message("reader stream setup", ce));
  for (int64_t c = t, i = 0; c < chunks && !failed->load(); c += n, ++i) {
    const int k = (int)(i & 1);
    if (pending[k] && (ce = cudaEventSynchronize(copied[k])) != cudaSuccess) {
      fail(TQ4_ERR_CUDA, cuda_message("cudaEventSynchronize", ce));
      break;
    }
    pending[k] = false;
    const int64_t off = c * kChunkBytes;
    const int64_t len = std::min(kChunkBytes, src->length - off);
    int64_t got = 0;
    while (got < len) {
      const ssize_t r = pread(fd, static_cast<char*>(slot[k]) + got, (size_t)(len - got),
                              (off_t)(src->offset + off + got));
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) {
        fail(TQ4_ERR_IO, r < 0 ? "reading " + src->path + ": " + strerror(errno)
                               : src->path + " ended before the external data range");
        break;
      }
      got += r;
    }
    if (got < len) break;
    ce = cudaMemcpyAsync(dst + off, slot[k], (size_t)len, cudaMemcpyHostToDevice, stream);
    if (ce == cudaSuccess) ce = cudaEventRecord(copied[k], stream);
    if (ce != cudaSuccess) {
      fail(TQ4_ERR_CUDA, cuda_message("chunk copy to the device", ce));
      break;
    }
    pending[k] = true;
  }
  // Every copy out of the pinned buffers has finished before the next read may reuse them.
  if (stream) {
    ce = cudaStreamSynchronize(stream);
    if (ce != cudaSuccess) fail(TQ4_ERR_CUDA, cuda_message("cudaStreamSynchronize", ce));
    cudaStreamDestroy(stream);
  }
  for (int k = 0; k < 2; ++k)
    if (copied[k]) cudaEventDestroy(copied[k]);
}

tq4_status read_file_to_device(void* dst, const Source& src, int device) {
  const int fd = open(src.path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    set_error("MatMulNBits: cannot open %s: %s", src.path.c_str(), strerror(errno));
    return TQ4_ERR_IO;
  }
  posix_fadvise(fd, (off_t)src.offset, (off_t)src.length, POSIX_FADV_SEQUENTIAL);
  const int64_t chunks = (src.length + kChunkBytes - 1) / kChunkBytes;
  const int hw = (int)std::max(1u, std::thread::hardware_concurrency());
  const int n = (int)std::min<int64_t>(chunks, std::min(kMaxReaders, hw));
  std::atomic<bool> failed{false};
  std::vector<ReadError> errs(n);
  std::vector<std::thread> readers;
  char* out = static_cast<char*>(dst);
  Staging& pool = staging();
  std::lock_guard<std::mutex> lock(pool.mu);
  for (int t = 0; t < n && !failed.load(); ++t) {
    for (int k = 0; k < 2; ++k) {
      if (pool.slot[t][k]) continue;
      const cudaError_t ce = cudaHostAlloc(&pool.slot[t][k], (size_t)kChunkBytes, cudaHostAllocPortable);
      if (ce != cudaSuccess) {
        pool.slot[t][k] = nullptr;
        errs[0].code = ce == cudaErrorMemoryAllocation ? TQ4_ERR_OUT_OF_MEMORY : TQ4_ERR_CUDA;
        errs[0].msg = cuda_message("pinned staging allocation", ce);
        failed.store(true);
        break;
      }
    }
  }
  try {
    for (int t = 1; t < n && !failed.load(); ++t)
      readers.emplace_back(read_chunks, fd, &src, out, device, t, n, chunks, pool.slot[t], &failed, &errs[t]);
  } catch (const std::exception& e) {
    // Chunks of a reader that did not start would be missing: stop the others.
    errs[0].code = TQ4_ERR_IO;
    errs[0].msg = std::string("cannot start a reader thread: ") + e.what();
    failed.store(true);
  }
  if (!failed.load()) read_chunks(fd, &src, out, device, 0, n, chunks, pool.slot[0], &failed, &errs[0]);
  for (auto& r : readers) r.join();
  close(fd);
  for (const ReadError& e : errs) {
    if (e.code != TQ4_OK) {
      set_error("MatMulNBits: %s", e.msg.c_str());
      return e.code;
    }
  }
  return TQ4_OK;
}

}  // namespace

tq4_status resolve_source(const tq4_source* in, int64_t expect, const char* what, Source* out) {
  *out = Source();
  if (!in || (!in->path && !in->data)) {
    set_error("MatMulNBits: %s is required", what);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (!in->path) {
    if (in->length != -1 && in->length != expect) {
      set_error("MatMulNBits: %s has %lld bytes, expected %lld", what, (long long)in->length,
                (long long)expect);
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    out->data = in->data;
    out->length = expect;
    return TQ4_OK;
  }
  struct stat sb;
  if (stat(in->path, &sb) != 0) {
    set_error("MatMulNBits: cannot read the external data of %s, %s: %s", what, in->path,
              strerror(errno));
    return TQ4_ERR_IO;
  }
  if (!S_ISREG(sb.st_mode)) {
    set_error("MatMulNBits: the external data of %s, %s, is not a regular file", what, in->path);
    return TQ4_ERR_IO;
  }
  const int64_t size = (int64_t)sb.st_size;
  if (in->offset < 0 || in->offset > size || in->length < -1) {
    set_error("MatMulNBits: external data of %s: offset %lld, length %lld outside %s (%lld bytes)",
              what, (long long)in->offset, (long long)in->length, in->path, (long long)size);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  // Without a length, the data runs to the end of the file (ops.ex:686-690).
  const int64_t length = in->length < 0 ? size - in->offset : in->length;
  if (length > size - in->offset) {
    set_error("MatMulNBits: external data of %s runs past the end of %s: offset %lld + length %lld > %lld bytes",
              what, in->path, (long long)in->offset, (long long)length, (long long)size);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (length != expect) {
    set_error("MatMulNBits: %s has %lld bytes in %s, expected %lld", what, (long long)length,
              in->path, (long long)expect);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  out->path = in->path;
  out->offset = in->offset;
  out->length = length;
  return TQ4_OK;
}

tq4_status fill_device(void* dst, const Source& src, int device, cudaStream_t st) {
  if (src.length == 0) return TQ4_OK;
  if (!src.path.empty()) return read_file_to_device(dst, src, device);
  TQ4_CUDA(cudaMemcpyAsync(dst, src.data, (size_t)src.length, cudaMemcpyDefault, st));
  return TQ4_OK;
}

}  // namespace tq4
