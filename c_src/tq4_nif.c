/* Erlang NIF over libtq4 (include/tq4.h): the native half of Transmuter.CUDAQ4
 * (lib/transmuter/cuda_q4.ex), the CUDA backend of Transmuter's MatMulNBits and
 * GatherBlockQuantized operators (lib/transmuter/ops/quantized.ex:30-66 in the reference).
 *
 * Build on a host with Erlang/OTP (c_src/Makefile):
 *   make -C c_src ERTS_INCLUDE_DIR=$(erl -noshell -eval 'io:format("~s/erts-~s/include",
 *        [code:root_dir(), erlang:system_info(version)])' -s init stop)
 *
 * Terms:
 *   - A weight is a resource holding a tq4_weight*; the resource destructor destroys the handle
 *     when the BEAM drops the last reference.
 *   - Device buffers (A, bias, Y, row indices, dequantized output) are passed as integers: the
 *     device pointers of the caller's backend (for EXLA, its buffers' device pointers). Stream 0
 *     is the legacy default stream.
 *   - Dtypes are the integers of tq4_dtype; zero-point kinds those of tq4_zp_kind.
 *   - Every call returns ok / {ok, Term} or {error, Message} with libtq4's message; none aborts.
 *
 * Scheduling: weight creation copies to the GPU and synchronizes, so it runs on a dirty I/O
 * scheduler. The compute entry points only enqueue work and return in microseconds.
 *
 * matmul_noalloc shares one static scratch array per device across all its calls: two of its
 * calls whose kernels overlap on the GPU race on that array. This NIF therefore serializes the
 * enqueue of noalloc calls with one mutex per device, and the caller must issue every noalloc
 * call of a device on one stream (so the GPU runs them in enqueue order). Concurrent callers on
 * several streams use matmul, whose scratch is per stream. */
#include <erl_nif.h>
#include <string.h>

#include "tq4.h"

#define TQ4_NIF_MAX_DEVICES 64
#define TQ4_NIF_MAX_MERGE 64

static ErlNifResourceType* WEIGHT;
static ErlNifMutex* NOALLOC_LOCK[TQ4_NIF_MAX_DEVICES];

typedef struct {
  tq4_weight* w;
  int device;
} weight_res;

static void weight_dtor(ErlNifEnv* env, void* obj) {
  (void)env;
  weight_res* r = (weight_res*)obj;
  if (r->w) tq4_weight_destroy(r->w);
  r->w = NULL;
}

static int load(ErlNifEnv* env, void** priv, ERL_NIF_TERM info) {
  (void)priv;
  (void)info;
  WEIGHT = enif_open_resource_type(env, NULL, "tq4_weight", weight_dtor, ERL_NIF_RT_CREATE, NULL);
  if (!WEIGHT) return 1;
  for (int d = 0; d < TQ4_NIF_MAX_DEVICES; ++d) {
    NOALLOC_LOCK[d] = enif_mutex_create("tq4_noalloc");
    if (!NOALLOC_LOCK[d]) return 1;
  }
  return 0;
}

static void unload(ErlNifEnv* env, void* priv) {
  (void)env;
  (void)priv;
  for (int d = 0; d < TQ4_NIF_MAX_DEVICES; ++d)
    if (NOALLOC_LOCK[d]) enif_mutex_destroy(NOALLOC_LOCK[d]);
}

static ERL_NIF_TERM error(ErlNifEnv* env) {
  char msg[512];
  tq4_last_error(msg, sizeof msg);
  return enif_make_tuple2(env, enif_make_atom(env, "error"), enif_make_string(env, msg, ERL_NIF_LATIN1));
}

static ERL_NIF_TERM ok_resource(ErlNifEnv* env, weight_res* r) {
  ERL_NIF_TERM ref = enif_make_resource(env, r);
  enif_release_resource(r);
  return enif_make_tuple2(env, enif_make_atom(env, "ok"), ref);
}

/* The description from argv[0..8]: K, N, Bits, BlockSize, ScaleDtype, ZpKind, ZpDtype,
 * DequantDtype, Signed (0 for u8 data, 1 for s8 data). */
static int get_desc(ErlNifEnv* env, const ERL_NIF_TERM argv[], tq4_weight_desc* d) {
  ErlNifSInt64 k, n;
  int bits, bs, sd, zk, zd, dd, sg;
  if (!enif_get_int64(env, argv[0], &k) || !enif_get_int64(env, argv[1], &n) ||
      !enif_get_int(env, argv[2], &bits) || !enif_get_int(env, argv[3], &bs) ||
      !enif_get_int(env, argv[4], &sd) || !enif_get_int(env, argv[5], &zk) ||
      !enif_get_int(env, argv[6], &zd) || !enif_get_int(env, argv[7], &dd) ||
      !enif_get_int(env, argv[8], &sg))
    return 0;
  memset(d, 0, sizeof *d);
  d->K = k;
  d->N = n;
  d->bits = bits;
  d->block_size = bs;
  d->scale_dtype = (tq4_dtype)sd;
  d->zp_kind = (tq4_zp_kind)zk;
  d->zp_dtype = (tq4_dtype)zd;
  d->dequant_dtype = (tq4_dtype)dd;
  d->b_signed = sg;
  return 1;
}

/* An input term: a binary (the bytes in memory) or {Path, Offset, Length} (a range of an ONNX
 * external-data file; Length -1 reads to the end of the file). */
static int get_source(ErlNifEnv* env, ERL_NIF_TERM t, tq4_source* src, char* path, unsigned cap) {
  ErlNifBinary bin;
  const ERL_NIF_TERM* tup;
  int arity;
  ErlNifSInt64 off, len;
  memset(src, 0, sizeof *src);
  if (enif_inspect_binary(env, t, &bin)) {
    src->data = bin.data;
    src->length = (int64_t)bin.size;
    return 1;
  }
  if (!enif_get_tuple(env, t, &arity, &tup) || arity != 3 ||
      enif_get_string(env, tup[0], path, cap, ERL_NIF_LATIN1) <= 0 || !enif_get_int64(env, tup[1], &off) ||
      !enif_get_int64(env, tup[2], &len))
    return 0;
  src->path = path;
  src->offset = off;
  src->length = len;
  return 1;
}

/* weight_create(K, N, Bits, BlockSize, ScaleDtype, ZpKind, ZpDtype, DequantDtype, Signed,
 *               B, Scales, Zp | nil, Device) -> {ok, Ref} | {error, Msg}
 * B, Scales and Zp are binaries (host bytes), or {Path, Offset, Length} file ranges, in which
 * case tq4_weight_create_from streams them to the GPU without reading them whole into the BEAM
 * (Transmuter.DeferredTensor, lib/transmuter/deferred_tensor.ex). */
static ERL_NIF_TERM weight_create(ErlNifEnv* env, int argc, const ERL_NIF_TERM argv[]) {
  (void)argc;
  tq4_weight_desc d;
  tq4_source b, s, z;
  char pb[4096], ps[4096], pz[4096];
  int dev;
  if (!get_desc(env, argv, &d) || !get_source(env, argv[9], &b, pb, sizeof pb) ||
      !get_source(env, argv[10], &s, ps, sizeof ps) || !enif_get_int(env, argv[12], &dev))
    return enif_make_badarg(env);
  const int has_zp = get_source(env, argv[11], &z, pz, sizeof pz);
  weight_res* r = enif_alloc_resource(WEIGHT, sizeof(weight_res));
  r->w = NULL;
  r->device = dev;
  tq4_status st;
  if (b.path || s.path || (has_zp && z.path))
    st = tq4_weight_create_from(&d, &b, &s, has_zp ? &z : NULL, dev, &r->w);
  else
    st = tq4_weight_create(&d, b.data, b.length, s.data, has_zp ? z.data : NULL, dev, &r->w);
  if (st != TQ4_OK) {
    enif_release_resource(r);
    return error(env);
  }
  return ok_resource(env, r);
}

/* weight_merge([Ref, ...]) -> {ok, Ref} | {error, Msg}: sibling MatMulNBits weights concatenated
 * along N (tq4_weight_merge; the packed form of Fusion.matmuls/2). The parts stay valid. */
static ERL_NIF_TERM weight_merge(ErlNifEnv* env, int argc, const ERL_NIF_TERM argv[]) {
  (void)argc;
  const tq4_weight* parts[TQ4_NIF_MAX_MERGE];
  unsigned count;
  ERL_NIF_TERM list = argv[0], head;
  if (!enif_get_list_length(env, list, &count) || count < 1 || count > TQ4_NIF_MAX_MERGE)
    return enif_make_badarg(env);
  int device = 0;
  for (unsigned i = 0; i < count; ++i) {
    weight_res* p;
    if (!enif_get_list_cell(env, list, &head, &list) || !enif_get_resource(env, head, WEIGHT, (void**)&p) || !p->w)
      return enif_make_badarg(env);
    parts[i] = p->w;
    device = p->device;
  }
  weight_res* r = enif_alloc_resource(WEIGHT, sizeof(weight_res));
  r->w = NULL;
  r->device = device;
  if (tq4_weight_merge(parts, (int)count, &r->w) != TQ4_OK) {
    enif_release_resource(r);
    return error(env);
  }
  return ok_resource(env, r);
}

/* The arguments of matmul and matmul_noalloc: Ref, APtr, M, ADtype, BiasPtr | 0, BiasDtype, YPtr,
 * YDtype, StreamPtr | 0. */
typedef struct {
  weight_res* r;
  ErlNifUInt64 a, bias, y, stream;
  ErlNifSInt64 m;
  int at, bt, yt;
} matmul_args;

static int get_matmul_args(ErlNifEnv* env, const ERL_NIF_TERM argv[], matmul_args* x) {
  return enif_get_resource(env, argv[0], WEIGHT, (void**)&x->r) && x->r->w && enif_get_uint64(env, argv[1], &x->a) &&
         enif_get_int64(env, argv[2], &x->m) && enif_get_int(env, argv[3], &x->at) &&
         enif_get_uint64(env, argv[4], &x->bias) && enif_get_int(env, argv[5], &x->bt) &&
         enif_get_uint64(env, argv[6], &x->y) && enif_get_int(env, argv[7], &x->yt) &&
         enif_get_uint64(env, argv[8], &x->stream);
}

/* matmul(...) -> ok | {error, Msg}: Y[M, N] = A . W^T (+ bias), the MatMulNBits clause
 * (quantized.ex:30-46). Enqueues on the stream and returns. */
static ERL_NIF_TERM matmul(ErlNifEnv* env, int argc, const ERL_NIF_TERM argv[]) {
  (void)argc;
  matmul_args x;
  if (!get_matmul_args(env, argv, &x)) return enif_make_badarg(env);
  if (tq4_matmul(x.r->w, (const void*)(uintptr_t)x.a, x.m, (tq4_dtype)x.at, x.bias ? (const void*)(uintptr_t)x.bias : NULL,
                 (tq4_dtype)x.bt, (void*)(uintptr_t)x.y, (tq4_dtype)x.yt, (void*)(uintptr_t)x.stream) != TQ4_OK)
    return error(env);
  return enif_make_atom(env, "ok");
}

/* matmul_noalloc(...) -> ok | {error, Msg}: the same for M <= 16 without any device allocation
 * (for a BEAM beside EXLA's client, which reserves most device memory up front). Its enqueue is
 * serialized per device; the caller keeps every noalloc call of a device on one stream. */
static ERL_NIF_TERM matmul_noalloc(ErlNifEnv* env, int argc, const ERL_NIF_TERM argv[]) {
  (void)argc;
  matmul_args x;
  if (!get_matmul_args(env, argv, &x) || x.r->device < 0 || x.r->device >= TQ4_NIF_MAX_DEVICES)
    return enif_make_badarg(env);
  enif_mutex_lock(NOALLOC_LOCK[x.r->device]);
  const tq4_status st = tq4_matmul_noalloc(
      x.r->w, (const void*)(uintptr_t)x.a, x.m, (tq4_dtype)x.at, x.bias ? (const void*)(uintptr_t)x.bias : NULL,
      (tq4_dtype)x.bt, (void*)(uintptr_t)x.y, (tq4_dtype)x.yt, (void*)(uintptr_t)x.stream);
  enif_mutex_unlock(NOALLOC_LOCK[x.r->device]);
  return st == TQ4_OK ? enif_make_atom(env, "ok") : error(env);
}

/* dequantize(Ref, OutPtr, StreamPtr | 0) -> ok | {error, Msg}: the {N, K} weight in its
 * dequantize type, bit for bit dequantize_weight/4 (quantized.ex:234-240). */
static ERL_NIF_TERM dequantize(ErlNifEnv* env, int argc, const ERL_NIF_TERM argv[]) {
  (void)argc;
  weight_res* r;
  ErlNifUInt64 out, stream;
  if (!enif_get_resource(env, argv[0], WEIGHT, (void**)&r) || !r->w || !enif_get_uint64(env, argv[1], &out) ||
      !enif_get_uint64(env, argv[2], &stream))
    return enif_make_badarg(env);
  if (tq4_dequantize(r->w, (void*)(uintptr_t)out, (void*)(uintptr_t)stream) != TQ4_OK) return error(env);
  return enif_make_atom(env, "ok");
}

/* gather_rows(Ref, IndicesPtr, Count, OutPtr, StreamPtr | 0) -> ok | {error, Msg}: rows of a
 * quantized table, dequantized (GatherBlockQuantized, quantized.ex:49-66). Indices are s64 on
 * the device; an index outside the table sets the device status (device_status/1). */
static ERL_NIF_TERM gather_rows(ErlNifEnv* env, int argc, const ERL_NIF_TERM argv[]) {
  (void)argc;
  weight_res* r;
  ErlNifUInt64 idx, out, stream;
  ErlNifSInt64 count;
  if (!enif_get_resource(env, argv[0], WEIGHT, (void**)&r) || !r->w || !enif_get_uint64(env, argv[1], &idx) ||
      !enif_get_int64(env, argv[2], &count) || !enif_get_uint64(env, argv[3], &out) ||
      !enif_get_uint64(env, argv[4], &stream))
    return enif_make_badarg(env);
  if (tq4_gather_rows(r->w, (const int64_t*)(uintptr_t)idx, count, (void*)(uintptr_t)out,
                      (void*)(uintptr_t)stream) != TQ4_OK)
    return error(env);
  return enif_make_atom(env, "ok");
}

/* device_status(Device) -> {ok, Code} | {error, Msg}: reads and clears the status word that
 * the kernels' bounded waits and argument checks write (0: no error). Synchronizes the device,
 * so it runs on a dirty scheduler. */
static ERL_NIF_TERM device_status(ErlNifEnv* env, int argc, const ERL_NIF_TERM argv[]) {
  (void)argc;
  int dev;
  int32_t code = 0;
  if (!enif_get_int(env, argv[0], &dev)) return enif_make_badarg(env);
  if (tq4_device_status(dev, &code) != TQ4_OK) return error(env);
  return enif_make_tuple2(env, enif_make_atom(env, "ok"), enif_make_int(env, code));
}

static ErlNifFunc funcs[] = {
    {"weight_create", 13, weight_create, ERL_NIF_DIRTY_JOB_IO_BOUND},
    {"weight_merge", 1, weight_merge, ERL_NIF_DIRTY_JOB_IO_BOUND},
    {"matmul", 9, matmul, 0},
    {"matmul_noalloc", 9, matmul_noalloc, 0},
    {"dequantize", 3, dequantize, 0},
    {"gather_rows", 5, gather_rows, 0},
    {"device_status", 1, device_status, ERL_NIF_DIRTY_JOB_IO_BOUND},
};

ERL_NIF_INIT(Elixir.Transmuter.CUDAQ4.NIF, funcs, load, NULL, NULL, unload)
