// The extern "C" entry points of include/tq4.h: argument checks, handle lifecycle, dispatch to
// the kernels. Errors become status codes plus a thread-local message, in the spirit of the
// reference's ArgumentError raises (quantized.ex:33-34) that run_nodes wraps with the op name
// and shapes (lib/transmuter.ex:661-679).
#include <cstdlib>
#include <cstdarg>

#include "internal.cuh"
#include "rows.cuh"

namespace tq4 {

static thread_local std::string t_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

void clear_error() { t_last_error.clear(); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("TQ4_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

void free_workspaces(Weight& w);

static bool is_float(tq4_dtype t) { return t == TQ4_F32 || t == TQ4_F16 || t == TQ4_BF16; }

static tq4_status check_desc(const tq4_weight_desc* d) {
  if (!d) {
    set_error("MatMulNBits: null weight description");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (d->K <= 0 || d->N <= 0) {
    set_error("MatMulNBits: K and N must be positive (K=%lld, N=%lld)", (long long)d->K,
              (long long)d->N);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (d->bits != 2 && d->bits != 4 && d->bits != 8) {
    set_error("MatMulNBits: bits must be 2, 4 or 8, got %d", d->bits);
    return TQ4_ERR_UNSUPPORTED;
  }
  if (d->block_size < 16 || (d->block_size & (d->block_size - 1)) != 0) {
    set_error("MatMulNBits: block_size must be a power of two >= 16, got %d", d->block_size);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (!is_float(d->scale_dtype) || !is_float(d->dequant_dtype)) {
    set_error("MatMulNBits: scales and the dequantize type must be f32, f16 or bf16");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (d->zp_kind == TQ4_ZP_PACKED && d->zp_dtype != TQ4_U8 && d->zp_dtype != TQ4_S8) {
    set_error("MatMulNBits: packed zero points must be u8 or s8");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (d->b_signed != 0 && d->b_signed != 1) {
    set_error("MatMulNBits: b_signed must be 0 (u8 data) or 1 (s8 data), got %d", d->b_signed);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  // Signed data is stored as unsigned data with each value's top bit flipped and every zero
  // point raised by 2^(bits-1) (the same differences q - z); that raised zero point must be exact.
  if (d->b_signed && d->zp_kind == TQ4_ZP_FLOAT) {
    set_error("MatMulNBits: signed data with float zero points is not supported");
    return TQ4_ERR_UNSUPPORTED;
  }
  if (d->b_signed && d->zp_kind == TQ4_ZP_PACKED && d->zp_dtype == TQ4_U8 && d->bits == 8 &&
      d->dequant_dtype == TQ4_BF16) {
    set_error("MatMulNBits: signed 8-bit data with u8 zero points cannot be dequantized in bf16");
    return TQ4_ERR_UNSUPPORTED;
  }
  if (d->zp_kind == TQ4_ZP_FLOAT && !is_float(d->zp_dtype)) {
    set_error("MatMulNBits: float zero points must be f32, f16 or bf16");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (d->zp_kind != TQ4_ZP_NONE && d->zp_kind != TQ4_ZP_PACKED && d->zp_kind != TQ4_ZP_FLOAT) {
    set_error("MatMulNBits: unknown zero-point kind %d", (int)d->zp_kind);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (d->K > (int64_t)1 << 30 || d->N > (int64_t)1 << 30) {
    set_error("MatMulNBits: K and N above 2^30 are not supported");
    return TQ4_ERR_UNSUPPORTED;
  }
  return TQ4_OK;
}

// A new handle for a checked description on `device` (made current by the caller): the layout,
// the handle's stream and its device buffers, zero-filled (padding rows and blocks stay zero).
static tq4_status layout_weight(const tq4_weight_desc* d, int device, const char* fn, tq4_weight** out) {
  tq4_weight* w = new tq4_weight();
  *out = w;
  w->desc = *d;
  w->device = device;
  w->blocks = (d->K + d->block_size - 1) / d->block_size;
  const int64_t G = 512 / d->bits;
  const int64_t k_valid = w->blocks * d->block_size;
  w->k_pad = (k_valid + G - 1) / G * G;
  w->row_bytes = w->k_pad * d->bits / 8;
  w->groups = w->row_bytes / 64;
  w->n_pad = (d->N + 127) / 128 * 128;
  const int64_t bp = (w->k_pad + d->block_size - 1) / d->block_size;
  w->blocks_pad = (bp + 7) / 8 * 8;
  while ((1 << w->bs_log2) < d->block_size) ++w->bs_log2;
  w->z_const = (float)(1 << (d->bits - 1));
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) == cudaSuccess) w->num_sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&w->stream, cudaStreamNonBlocking) != cudaSuccess) {
    set_error("%s: cudaStreamCreate failed", fn);
    return TQ4_ERR_CUDA;
  }
  const int tsz = dtype_size(d->dequant_dtype);
  TQ4_TRY(w->q.alloc(w->n_pad * w->row_bytes));
  TQ4_TRY(w->scales.alloc(w->n_pad * w->blocks_pad * tsz));
  if (d->zp_kind != TQ4_ZP_NONE) TQ4_TRY(w->zps.alloc(w->n_pad * w->blocks_pad * tsz));
  return TQ4_OK;
}

static tq4_status make_maps(tq4_weight* w) {
  TQ4_TRY(make_weight_maps(*w));
  TQ4_TRY(make_gemv_maps(*w));
  return make_rows_maps(*w);
}

// The handle of a checked description and resolved inputs, on `device`.
static tq4_status create_weight(const tq4_weight_desc* d, const Source& b, const Source& s,
                                const Source* z, int device, tq4_weight** out, const char* fn) {
  int ndev = 0;
  TQ4_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) {
    set_error("%s: device %d out of range (%d devices)", fn, device, ndev);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  int prev = 0;
  TQ4_CUDA(cudaGetDevice(&prev));
  TQ4_CUDA(cudaSetDevice(device));
  tq4_weight* w = nullptr;
  tq4_status st = layout_weight(d, device, fn, &w);
  if (st == TQ4_OK) st = prepare_weight(*w, b, s, z);
  if (st == TQ4_OK) st = make_maps(w);
  cudaSetDevice(prev);
  if (st != TQ4_OK) {
    tq4_weight_destroy(w);
    return st;
  }
  *out = w;
  return TQ4_OK;
}

// One handle over the rows of `parts` in order (tq4_weight_merge).
static tq4_status merge_handles(const tq4_weight* const* parts, int count, tq4_weight** out) {
  const tq4_weight_desc& d0 = parts[0]->desc;
  tq4_weight_desc d = d0;
  int64_t n = 0;
  for (int i = 0; i < count; ++i) {
    const tq4_weight* p = parts[i];
    const tq4_weight_desc& di = p->desc;
    if (di.K != d0.K || di.bits != d0.bits || di.block_size != d0.block_size || di.scale_dtype != d0.scale_dtype ||
        di.zp_kind != d0.zp_kind || (di.zp_kind != TQ4_ZP_NONE && di.zp_dtype != d0.zp_dtype) ||
        di.dequant_dtype != d0.dequant_dtype || di.b_signed != d0.b_signed || p->device != parts[0]->device) {
      set_error("tq4_weight_merge: part %d differs from part 0 (K, bits, block_size, scale or zero-point type, "
                "dequantize type, signedness or device)", i);
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    n += di.N;
  }
  d.N = n;
  TQ4_TRY(check_desc(&d));
  int prev = 0;
  TQ4_CUDA(cudaGetDevice(&prev));
  TQ4_CUDA(cudaSetDevice(parts[0]->device));
  tq4_weight* w = nullptr;
  tq4_status st = layout_weight(&d, parts[0]->device, "tq4_weight_merge", &w);
  if (st == TQ4_OK && cudaMemsetAsync(w->q.ptr, 0, w->q.bytes, w->stream) != cudaSuccess) st = TQ4_ERR_CUDA;
  if (st == TQ4_OK && cudaMemsetAsync(w->scales.ptr, 0, w->scales.bytes, w->stream) != cudaSuccess) st = TQ4_ERR_CUDA;
  if (st == TQ4_OK && w->zps.ptr && cudaMemsetAsync(w->zps.ptr, 0, w->zps.bytes, w->stream) != cudaSuccess)
    st = TQ4_ERR_CUDA;
  if (st == TQ4_ERR_CUDA) set_error("tq4_weight_merge: cudaMemsetAsync failed");
  if (st == TQ4_OK) st = merge_weight(*w, parts, count);
  if (st == TQ4_OK) st = make_maps(w);
  cudaSetDevice(prev);
  if (st != TQ4_OK) {
    tq4_weight_destroy(w);
    return st;
  }
  *out = w;
  return TQ4_OK;
}

}  // namespace tq4

using namespace tq4;

extern "C" {

const char* tq4_status_string(tq4_status s) {
  switch (s) {
    case TQ4_OK: return "ok";
    case TQ4_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TQ4_ERR_UNSUPPORTED: return "unsupported";
    case TQ4_ERR_CUDA: return "CUDA error";
    case TQ4_ERR_NCCL: return "NCCL error";
    case TQ4_ERR_OUT_OF_MEMORY: return "out of device memory";
    case TQ4_ERR_TIMEOUT: return "timed out";
    case TQ4_ERR_DEVICE: return "device-side error";
    case TQ4_ERR_IO: return "file error";
  }
  return "unknown status";
}

size_t tq4_last_error(char* buf, size_t len) {
  const std::string& e = t_last_error;
  if (buf && len > 0) {
    const size_t n = std::min(len - 1, e.size());
    memcpy(buf, e.data(), n);
    buf[n] = 0;
  }
  return e.size();
}

tq4_status tq4_weight_input_sizes(const tq4_weight_desc* d, int64_t* b_bytes, int64_t* scale_bytes,
                                  int64_t* zp_bytes) {
  clear_error();
  TQ4_TRY(check_desc(d));
  const int64_t blocks = (d->K + d->block_size - 1) / d->block_size;
  if (b_bytes) *b_bytes = d->N * blocks * d->block_size * d->bits / 8;
  if (scale_bytes) *scale_bytes = d->N * blocks * dtype_size(d->scale_dtype);
  if (zp_bytes) {
    *zp_bytes = 0;
    if (d->zp_kind == TQ4_ZP_PACKED) *zp_bytes = d->N * ((blocks * d->bits + 7) / 8);
    if (d->zp_kind == TQ4_ZP_FLOAT) *zp_bytes = d->N * blocks * dtype_size(d->zp_dtype);
  }
  return TQ4_OK;
}

tq4_status tq4_weight_create(const tq4_weight_desc* d, const void* b, int64_t b_bytes,
                             const void* scales, const void* zp, int device, tq4_weight** out) {
  clear_error();
  if (!out) {
    set_error("tq4_weight_create: null output handle");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  *out = nullptr;
  TQ4_TRY(check_desc(d));
  int64_t need_b = 0;
  TQ4_TRY(tq4_weight_input_sizes(d, &need_b, nullptr, nullptr));
  if (!b || !scales) {
    set_error("MatMulNBits: B and scales are required");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (b_bytes != need_b) {
    set_error("MatMulNBits: B has %lld bytes, expected N*ceil(K/block_size)*block_size*bits/8 = %lld",
              (long long)b_bytes, (long long)need_b);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (d->zp_kind != TQ4_ZP_NONE && !zp) {
    set_error("MatMulNBits: zero points declared but not given");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  int64_t s_bytes = 0, z_bytes = 0;
  TQ4_TRY(tq4_weight_input_sizes(d, nullptr, &s_bytes, &z_bytes));
  Source bs, ss, zs;
  bs.data = b;
  bs.length = need_b;
  ss.data = scales;
  ss.length = s_bytes;
  zs.data = zp;
  zs.length = z_bytes;
  return create_weight(d, bs, ss, d->zp_kind != TQ4_ZP_NONE ? &zs : nullptr, device, out,
                       "tq4_weight_create");
}

tq4_status tq4_weight_create_from(const tq4_weight_desc* d, const tq4_source* b,
                                  const tq4_source* scales, const tq4_source* zp, int device,
                                  tq4_weight** out) {
  clear_error();
  if (!out) {
    set_error("tq4_weight_create_from: null output handle");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  *out = nullptr;
  TQ4_TRY(check_desc(d));
  int64_t b_bytes = 0, s_bytes = 0, z_bytes = 0;
  TQ4_TRY(tq4_weight_input_sizes(d, &b_bytes, &s_bytes, &z_bytes));
  Source bs, ss, zs;
  TQ4_TRY(resolve_source(b, b_bytes, "B", &bs));
  TQ4_TRY(resolve_source(scales, s_bytes, "scales", &ss));
  if (d->zp_kind != TQ4_ZP_NONE) {
    if (!zp) {
      set_error("MatMulNBits: zero points declared but not given");
      return TQ4_ERR_INVALID_ARGUMENT;
    }
    TQ4_TRY(resolve_source(zp, z_bytes, "zero points", &zs));
  }
  return create_weight(d, bs, ss, d->zp_kind != TQ4_ZP_NONE ? &zs : nullptr, device, out,
                       "tq4_weight_create_from");
}

tq4_status tq4_weight_destroy(tq4_weight* w) {
  if (!w) return TQ4_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(w->device);
  free_workspaces(*w);
  w->q.release();
  w->scales.release();
  w->zps.release();
  if (w->stream) cudaStreamDestroy(w->stream);
  delete w;
  cudaSetDevice(prev);
  return TQ4_OK;
}

tq4_status tq4_weight_merge(const tq4_weight* const* parts, int count, tq4_weight** out) {
  clear_error();
  if (!out || !parts || count < 1) {
    set_error("tq4_weight_merge: null output, no parts");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  *out = nullptr;
  for (int i = 0; i < count; ++i)
    if (!parts[i]) {
      set_error("tq4_weight_merge: part %d is null", i);
      return TQ4_ERR_INVALID_ARGUMENT;
    }
  return merge_handles(parts, count, out);
}

tq4_status tq4_weight_info(const tq4_weight* w, tq4_weight_desc* d, int64_t* device_bytes) {
  clear_error();
  if (!w) {
    set_error("tq4_weight_info: null handle");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (d) *d = w->desc;
  if (device_bytes) *device_bytes = w->q.bytes + w->scales.bytes + w->zps.bytes;
  return TQ4_OK;
}

// RAII switch to the handle's device for the duration of a call.
tq4_status tq4_matmul(const tq4_weight* w, const void* a, int64_t m, tq4_dtype a_t,
                      const void* bias, tq4_dtype bias_t, void* y, tq4_dtype y_t, void* stream) {
  clear_error();
  if (!w) {
    set_error("MatMulNBits: null weight handle");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (m < 0 || m > ((int64_t)1 << 31) / std::max<int64_t>(1, w->desc.K)) {
    set_error("MatMulNBits: M=%lld out of range", (long long)m);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (!is_float(a_t) || !is_float(y_t) || (bias && !is_float(bias_t))) {
    set_error("MatMulNBits: A, bias and Y must be f32, f16 or bf16");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (m == 0) return TQ4_OK;
  if (!a || !y) {
    set_error("MatMulNBits: null A or Y");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceGuard guard(w->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return run_matmul(*w, a, m, a_t, bias, bias_t, y, y_t, w->desc.N, st);
}

tq4_status tq4_dequantize(const tq4_weight* w, void* out, void* stream) {
  clear_error();
  if (!w || !out) {
    set_error("tq4_dequantize: null handle or output");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceGuard guard(w->device);
  return run_dequant(*w, nullptr, w->desc.N, out, static_cast<cudaStream_t>(stream));
}

tq4_status tq4_gather_rows(const tq4_weight* w, const int64_t* indices, int64_t count, void* out,
                           void* stream) {
  clear_error();
  if (!w || (count > 0 && (!indices || !out)) || count < 0) {
    set_error("GatherBlockQuantized: null handle, indices or output");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceGuard guard(w->device);
  return run_dequant(*w, indices, count, out, static_cast<cudaStream_t>(stream));
}

tq4_status tq4_set_wait_limit(int device, int64_t cycles) {
  clear_error();
  int ndev = 0;
  TQ4_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) {
    set_error("tq4_set_wait_limit: device %d out of range (%d devices)", device, ndev);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  if (cycles < 0 || (cycles > 0 && cycles < 1000)) {
    set_error("tq4_set_wait_limit: %lld cycles (0 for the default, else at least 1000)", (long long)cycles);
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceGuard guard(device);
  const long long v = cycles == 0 ? 2000000000LL : (long long)cycles;
  TQ4_CUDA(cudaDeviceSynchronize());  // no kernel of this device waits while the limit changes
  TQ4_CUDA(cudaMemcpyToSymbol(g_wait_cycles, &v, sizeof(v)));
  return TQ4_OK;
}

tq4_status tq4_device_status(int device, int32_t* code) {
  clear_error();
  if (!code) {
    set_error("tq4_device_status: null output");
    return TQ4_ERR_INVALID_ARGUMENT;
  }
  DeviceGuard guard(device);
  TQ4_CUDA(cudaDeviceSynchronize());
  int32_t v = 0;
  TQ4_CUDA(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)));
  const int32_t zero = 0;
  TQ4_CUDA(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)));
  *code = v;
  return TQ4_OK;
}

}  // extern "C"
