// Prefill-shaped MatMulNBits calls (M > 16).
#include "internal.cuh"

namespace tq4 {

// Rows of A in slices of 16 through the fused GEMV kernel.
static tq4_status run_gemm_by_slices(const Weight& w, const void* a, int64_t m, tq4_dtype a_t,
                                     const void* bias, tq4_dtype bias_t, void* y, tq4_dtype y_t,
                                     int64_t ldy, cudaStream_t st) {
  const int as = dtype_size(a_t), ys = dtype_size(y_t);
  for (int64_t r = 0; r < m; r += 16) {
    const int64_t rows = std::min<int64_t>(16, m - r);
    TQ4_TRY(run_gemv(w, static_cast<const uint8_t*>(a) + r * w.desc.K * as, rows, a_t, bias,
                     bias_t, static_cast<uint8_t*>(y) + r * ldy * ys, y_t, ldy, st));
  }
  return TQ4_OK;
}

tq4_status run_gemm(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                    tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  return run_gemm_by_slices(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
}

tq4_status run_matmul(const Weight& w, const void* a, int64_t m, tq4_dtype a_t, const void* bias,
                      tq4_dtype bias_t, void* y, tq4_dtype y_t, int64_t ldy, cudaStream_t st) {
  if (m <= 16) return run_gemv(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
  return run_gemm(w, a, m, a_t, bias, bias_t, y, y_t, ldy, st);
}

}  // namespace tq4
