/*
 * tq4 — B200-native (sm_100a) MatMulNBits for Transmuter.
 *
 * This is the C ABI that Transmuter's MatMulNBits operator binds (through an Erlang NIF in the
 * reference's world, through ctypes in this repository's tests). Every entry point takes plain
 * pointers and sizes, returns a tq4_status, and never aborts or traps: a failure leaves a
 * message for tq4_last_error() on the calling thread.
 *
 * The operator (georgeguimaraes/transmuter, lib/transmuter/ops/quantized.ex:30-46) is
 *     Y[..., N] = A[..., K] . W^T (+ bias)
 * where W {N, K} is dequantized from B u8 [N, blocks, block_size*bits/8] (bits values per byte,
 * lowest bits first), per-block scales [N*blocks] and optional zero points (absent -> 2^(bits-1),
 * packed bits [N, ceil(blocks*bits/8)], or floats [N*blocks]): W = (q - zero) * scale in a float
 * type T, one rounding per step, then sliced to K columns (quantized.ex:234-240,306-325;
 * packed.ex:9-36). `accuracy_level` is not an input: the reference never reads it.
 *
 * Pointers named "device" must be CUDA device (or managed) memory of the handle's device; pointers
 * to tq4_weight_create may be host or device memory. Streams are cudaStream_t passed as void*
 * (NULL = the legacy default stream).
 */
#ifndef TQ4_H
#define TQ4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  TQ4_OK = 0,
  TQ4_ERR_INVALID_ARGUMENT = 1, /* bad sizes, null pointers, inconsistent attributes */
  TQ4_ERR_UNSUPPORTED = 2,      /* a valid operator the library does not implement (g_idx, bits) */
  TQ4_ERR_CUDA = 3,             /* a CUDA runtime/driver call failed */
  TQ4_ERR_NCCL = 4,             /* an NCCL call failed or NCCL is not loadable */
  TQ4_ERR_OUT_OF_MEMORY = 5,
  TQ4_ERR_TIMEOUT = 6,          /* a bounded wait (device or host) ran out */
  TQ4_ERR_DEVICE = 7,           /* a kernel reported an error through the device status word */
  TQ4_ERR_IO = 8                /* a file given to tq4_weight_create_from cannot be opened or read */
} tq4_status;

typedef enum { TQ4_F32 = 0, TQ4_F16 = 1, TQ4_BF16 = 2, TQ4_U8 = 3, TQ4_S8 = 4 } tq4_dtype;

/* Zero points of block_zero_points/5 (quantized.ex:306-325). */
typedef enum { TQ4_ZP_NONE = 0, TQ4_ZP_PACKED = 1, TQ4_ZP_FLOAT = 2 } tq4_zp_kind;

/* The attributes and input types of one MatMulNBits node.
 *   K, N, bits, block_size: the node attributes (quantized.ex:226-228; bits 2, 4 or 8;
 *       block_size a power of two >= 16).
 *   scale_dtype: type of the scales input (F32, F16 or BF16), N*ceil(K/block_size) values.
 *   zp_kind / zp_dtype: zero points; zp_dtype is U8 or S8 for packed zero points (N rows of
 *       ceil(blocks*bits/8) bytes; S8 values are sign extended like signed data) or the float
 *       type of float zero points (N*blocks values).
 *   dequant_dtype: the float type T the weight is dequantized in. In the graph it is A's type
 *       (quantized.ex:42); for a moved model it is the scales' type after :compute_type
 *       (lib/transmuter.ex:1230-1233).
 *   b_signed: 0 for u8 data (MatMulNBits' B is always u8). 1 for s8 data, as int4 and int2 exports
 *       of a GatherBlockQuantized table load it (quantized.ex:294-300): each value is sign
 *       extended and the default zero point is 0. Signed data takes no float zero points, and
 *       with u8 packed zero points not bits 8 with bf16 dequantization (the zero point plus
 *       2^(bits-1) that the handle stores would round). */
typedef struct {
  int64_t K;
  int64_t N;
  int32_t bits;
  int32_t block_size;
  tq4_dtype scale_dtype;
  tq4_zp_kind zp_kind;
  tq4_dtype zp_dtype;
  tq4_dtype dequant_dtype;
  int32_t b_signed;
} tq4_weight_desc;

typedef struct tq4_weight tq4_weight;
typedef struct tq4_comm tq4_comm;
typedef struct tq4_sharded tq4_sharded;

/* Bytes of each input that tq4_weight_create reads for `desc` (B, scales, zero points). */
tq4_status tq4_weight_input_sizes(const tq4_weight_desc* desc, int64_t* b_bytes,
                                  int64_t* scale_bytes, int64_t* zp_bytes);

/* Replaces the load-time weight builder of Transmuter.move/2 (lib/transmuter.ex:1104-1182,
 * dequantized_weight/6 at :1230-1240, and the EMLX packer lib/transmuter/emlx.ex:104-148):
 * copies B, scales and zero points once to `device` and keeps them packed there, in the
 * handle's own layout. `zp` may be NULL when desc->zp_kind is TQ4_ZP_NONE. Unlike packable?/2
 * (lib/transmuter.ex:1209-1225), a K that is not a multiple of block_size is accepted. */
tq4_status tq4_weight_create(const tq4_weight_desc* desc, const void* b, int64_t b_bytes,
                             const void* scales, const void* zp, int device, tq4_weight** out);

/* One input of tq4_weight_create_from: bytes in memory, or an initializer whose data an ONNX
 * model keeps in a file beside it (TensorProto data_location EXTERNAL, with the external_data
 * entries "location", "offset" and "length"; lib/transmuter/ops.ex:680-695). */
typedef struct {
  const void* data;   /* host or device memory; used when path is NULL */
  const char* path;   /* the file: the model's directory joined with "location" */
  int64_t offset;     /* "offset" (0 when the entry is absent) */
  int64_t length;     /* "length" in bytes; -1 when absent: from offset to the end of the file.
                         For data, its byte count (-1: the size the descriptor implies). */
} tq4_source;

/* tq4_weight_create with each input given as a tq4_source. Replaces the read of a deferred
 * initializer at move time (Transmuter.DeferredTensor.value/1, lib/transmuter/deferred_tensor.ex
 * :27, read by move/2 at lib/transmuter.ex:1159, and Ops.read_external/2 at ops.ex:680-695): the
 * file range streams to the device through a few pinned chunks, without a host copy of the
 * tensor. Each input's byte count must be the one the descriptor implies (tq4_weight_input_sizes).
 * A file that cannot be opened is TQ4_ERR_IO and a range past its end TQ4_ERR_INVALID_ARGUMENT,
 * both found before any device work; a read that fails later is TQ4_ERR_IO. `zp` may be NULL when
 * desc->zp_kind is TQ4_ZP_NONE. The handle is the one tq4_weight_create makes from the same
 * bytes. */
tq4_status tq4_weight_create_from(const tq4_weight_desc* desc, const tq4_source* b,
                                  const tq4_source* scales, const tq4_source* zp, int device,
                                  tq4_weight** out);

tq4_status tq4_weight_destroy(tq4_weight* w);

/* Merges sibling MatMulNBits weights along N, the packed form of Fusion.matmuls/2
 * (lib/transmuter/fusion.ex:430-540, which concatenates the moved float {N, K} weights of matmuls
 * that read one input, such as q, k and v, or gate and up, and adds a Split): a new handle whose
 * rows are the rows of parts[0], then parts[1], ..., N the sum of the parts' N. The parts must
 * share K, bits, block_size, the scale and zero-point types, the dequantize type and the device;
 * the copies stay on the device, and the parts remain valid (the caller destroys them). One call
 * on the merged handle gives every part's Y: columns [off_i, off_i + N_i) are part i's, off_i the
 * sum of the N before it (the Split). Its dequantized weight is the row concatenation of the
 * parts', bit for bit. */
tq4_status tq4_weight_merge(const tq4_weight* const* parts, int count, tq4_weight** out);

/* The handle's attributes and the device bytes it holds. */
tq4_status tq4_weight_info(const tq4_weight* w, tq4_weight_desc* desc, int64_t* device_bytes);

/* Replaces the MatMulNBits clause (quantized.ex:30-46) for a weight the handle holds:
 *   Y[M, N] = A[M, K] . W^T (+ bias[N]),  W = dequantize_weight(...) in desc.dequant_dtype.
 * A (a_dtype F32/F16/BF16), bias (bias_dtype; NULL for none) and Y (y_dtype) are device
 * pointers, row-major and dense. M >= 0 (M = 0 is a no-op). Calls with M <= 8 run the fused
 * unpack-dequant-GEMV kernel; larger M run the tensor-core GEMM, except that calls with
 * 9 <= M <= 16 it cannot take (bits other than 4, an A that is not 16-byte aligned) run the GEMV
 * too. */
tq4_status tq4_matmul(const tq4_weight* w, const void* a, int64_t m, tq4_dtype a_dtype,
                      const void* bias, tq4_dtype bias_dtype, void* y, tq4_dtype y_dtype,
                      void* stream);

/* tq4_matmul for M <= 16 that allocates no device memory. No counterpart in the reference: it
 * serves callers that cannot call cudaMalloc, such as a NIF sharing the GPU with EXLA's client
 * (which reserves most device memory up front) or a decode loop that must not risk the device
 * synchronization of cudaMalloc/cudaFree. Its split-K scratch is a static 4 MiB device array
 * (plus 64 KiB of counters), held on a GPU from the moment the library's device code is loaded
 * there until exit. With CUDA's default lazy module loading that is the first tq4 call on that
 * GPU, not the library load: make one tq4 call per GPU before another allocator reserves its
 * memory, or set CUDA_MODULE_LOADING=EAGER. A call that
 * would need more is rejected with TQ4_ERR_INVALID_ARGUMENT, and M > 16 with
 * TQ4_ERR_UNSUPPORTED. The first call on a device looks up the array's device address (make it
 * before any stream capture). Calls share the array: calls that overlap on the GPU race. */
tq4_status tq4_matmul_noalloc(const tq4_weight* w, const void* a, int64_t m, tq4_dtype a_dtype,
                              const void* bias, tq4_dtype bias_dtype, void* y, tq4_dtype y_dtype,
                              void* stream);

/* dequantize_weight/4 (quantized.ex:234-240) on the device: W[N, K] in desc.dequant_dtype,
 * bit-exact with the reference. `out` is a device pointer of N*K elements. */
tq4_status tq4_dequantize(const tq4_weight* w, void* out, void* stream);

/* GatherBlockQuantized (quantized.ex:49-66) over a handle's rows: out[i, :] = the dequantized
 * row indices[i] of W, for a table stored as a MatMulNBits weight (tied embeddings). indices
 * are int64 device values in [0, N); out is [count, K] in desc.dequant_dtype. */
tq4_status tq4_gather_rows(const tq4_weight* w, const int64_t* indices, int64_t count, void* out,
                           void* stream);

/* Reads and clears the device status word that bounded waits and device-side checks write.
 * Synchronizes the handle's device. *code = 0 when no kernel reported an error. Codes: 0x101-0x104
 * a tensor-core GEMM pipeline wait ran out, 0x105 a split-K counter was inconsistent, 0x106 a
 * peer's flag did not arrive (N-sharded calls), 0x107 a decode-attention copy, 0x108 the GEMV's
 * activation staging, 0x200 a device-side argument check (decoder positions).
 * Failure detection of the reference: test/support/hang_watchdog.exs:1-40 flags a call that makes
 * no progress; here every device wait gives up after a limit and reports instead. */
tq4_status tq4_device_status(int device, int32_t* code);

/* The limit of every bounded device wait on `device` (mbarrier waits of the GEMV, GEMM and
 * decoder kernels; the peer-flag waits of N-sharded calls), in SM clock cycles: 0 restores the
 * default of 2e9 (about one second at the B200's clocks), other values must be at least 1000.
 * Synchronizes the device first. Meant for failure tests and for watchdogs that must fire
 * sooner; a limit below a healthy call's own waits makes that call report a timeout. */
tq4_status tq4_set_wait_limit(int device, int64_t cycles);

/* Runs the peer-flag wait of the N-sharded kernels on `stream` against a flag that nothing ever
 * sets: after the device's wait limit the kernel gives up, reports 0x106 in the device status and
 * returns, and the context stays usable. A self-test of the timeout path (no counterpart in the
 * reference). */
tq4_status tq4_selftest_peer_wait(int device, void* stream);

/* The message of the last failure on the calling thread ("" when none). Returns the length
 * of the full message; at most len-1 bytes and a NUL are written to buf. */
size_t tq4_last_error(char* buf, size_t len);

const char* tq4_status_string(tq4_status status);

/* ---- N-sharded execution over NCCL (one process or thread per GPU) -------------------------
 * The weight is split along N (rows of B, scales and zero points); each rank computes its
 * columns of Y and an all-gather over NVLink assembles Y on every rank. No reference
 * counterpart exists (the reference has no device collective); it serves the 151936-column
 * lm_head and the Llama-shaped projections of the north star. */

#define TQ4_UNIQUE_ID_BYTES 128

/* Rank 0 makes the id and sends it to the other ranks by any host channel. */
tq4_status tq4_comm_unique_id(unsigned char id[TQ4_UNIQUE_ID_BYTES]);

/* Joins the communicator; waits at most timeout_ms for the other ranks (0 = 60000). */
tq4_status tq4_comm_create(const unsigned char id[TQ4_UNIQUE_ID_BYTES], int nranks, int rank,
                           int device, int timeout_ms, tq4_comm** out);

tq4_status tq4_comm_destroy(tq4_comm* comm);

/* Each rank owns share = ceil(N/P) rounded up to 16 rows: rows [rank*share, rank*share+share)
 * of the FULL B, scales and zero points (clipped to N; the last ranks may own fewer or none)
 * become this rank's handle. The inputs may be host or device memory. */
tq4_status tq4_sharded_create(const tq4_weight_desc* desc, const void* b, int64_t b_bytes,
                              const void* scales, const void* zp, tq4_comm* comm,
                              tq4_sharded** out);

/* tq4_sharded_create with each FULL input given as a tq4_source: a file range (ONNX external
 * data) is narrowed to this rank's rows, so each rank reads only its share of the file. */
tq4_status tq4_sharded_create_from(const tq4_weight_desc* desc, const tq4_source* b,
                                   const tq4_source* scales, const tq4_source* zp, tq4_comm* comm,
                                   tq4_sharded** out);

/* This rank's first row and row count. */
tq4_status tq4_sharded_rows(const tq4_sharded* s, int64_t* first, int64_t* count);

/* Y[M, N] on every rank: the local MatMulNBits on this rank's rows, then Y assembled on every rank.
 * M = 1 with 4-bit weights of at most 8 packed groups per row (the lm_head): each rank's GEMV
 * stores its columns straight into every rank's assembly buffer over NVLink, and one small kernel
 * exchanges an epoch flag per peer (bounded wait, device status 0x106 on timeout) and copies the
 * row into Y. Slices of 4 MB and more per rank: an NVLink exchange of the ranks' slices. Otherwise
 * (or where peer mapping is not available on every rank): NCCL's all-gather. A, bias (full N, or
 * NULL) and Y are device pointers on the comm's device. Every rank makes the same calls in the
 * same order; the first call of a new shape maps peer memory (a collective) and must come before
 * any stream capture. */
tq4_status tq4_sharded_matmul(const tq4_sharded* s, const void* a, int64_t m, tq4_dtype a_dtype,
                              const void* bias, tq4_dtype bias_dtype, void* y, tq4_dtype y_dtype,
                              void* stream);

tq4_status tq4_sharded_destroy(tq4_sharded* s);

#ifdef __cplusplus
}
#endif

#endif /* TQ4_H */
