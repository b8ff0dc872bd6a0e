// Host-side interface of the 32-row-unit M = 1 GEMV (gemv_rows.cu), shared with the dispatcher
// (gemv.cu) and the N-sharded push path (sharded.cu).
#pragma once

#include "internal.cuh"

namespace tq4 {

constexpr int kRowsMaxDst = 8;  // Y itself, or one assembly buffer per rank (at most 8 ranks)

// Where a call's outputs go: row n of the weight is Y column col0 + n of each destination; with
// `epoch` set (N-sharded calls) the outputs land in the half ((*epoch + 1) & 1) of every
// destination buffer, halves of half_elems elements.
struct RowsDst {
  void* y[kRowsMaxDst] = {};
  int ndst = 1;
  int64_t col0 = 0;
  const unsigned long long* epoch = nullptr;
  int64_t half_elems = 0;
};

// An RMSNorm of the f32 activation row before the product (the decoder's fused projections,
// rms_norm/4 of transformer.ex:1056-1069): a = x * rsqrt(mean(x^2) + eps) * w.
struct RowsNorm {
  const float* w = nullptr;
  float eps = 0.f;
};

// 4-bit weights whose unit descriptors were made (block_size <= 1024). Rows of more than 8 packed
// groups run K-sliced: each CTA takes one slice of 8 groups for the whole call, and the slices'
// partial rows are added in slice order by the last slice to finish a unit.
bool rows_eligible(const Weight& w);
// Slices of 8 packed groups per row (1 for rows of at most 8 groups).
int rows_slices(const Weight& w);
// Workspace floats and counters of a call (slice tickets, then one arrival counter per unit for
// K-sliced rows); both left as they were found (counters at zero).
int64_t rows_ws_floats(const Weight& w);
int64_t rows_counters(const Weight& w);
// The unit descriptors of a new handle (a no-op for handles the kernel does not take).
tq4_status make_rows_maps(Weight& w);
// Y = A . W^T (+ bias) for one activation row; `counter` is rows_counters(w) ints of device memory
// that are zero before the call and left at zero by it, `ws` rows_ws_floats(w) floats (per
// stream: calls that overlap must not share them). K-sliced rows take neither the RMSNorm
// prologue nor several destinations.
tq4_status run_gemv_rows(const Weight& w, const void* a, tq4_dtype a_t, const void* bias, tq4_dtype bias_t,
                         tq4_dtype y_t, const RowsDst& dst, int* counter, cudaStream_t st,
                         const RowsNorm* norm = nullptr, float* ws = nullptr);

}  // namespace tq4
