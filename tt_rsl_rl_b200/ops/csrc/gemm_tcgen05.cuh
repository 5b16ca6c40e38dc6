// Host-visible interface of the tcgen05 GEMM used by every MLP layer (forward, data-gradient, weight-gradient).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rlb {

// out[M, N] = sum_k A(m, k) * B(n, k)   (bf16 operands, fp32 accumulation in TMEM)
//
// Operand storage (row-major with leading dimension in elements):
//   A K-major : A(m, k) = a[m * lda + k]          A MN-major : A(m, k) = a[k * lda + m]
//   B K-major : B(n, k) = b[n * ldb + k]          B MN-major : B(n, k) = b[k * ldb + n]
// The leading dimension times 2 bytes must be a multiple of 16 (TMA stride rule); extents need not be.
// bf16 outputs (and the bf16 aux input) need 16-byte aligned bases and ldo, ld_aux multiples of 8. They leave through
// TMA stores in 16-byte column groups: columns [N, N rounded up to 8) of each output row receive zeros (the
// accumulator columns past N are zero), columns beyond are untouched.
enum GemmEpilogue : int {
  kEpiF32 = 0,         // out fp32 = acc (+ bias[n])
  kEpiBiasEluBf16 = 1, // out bf16 = elu(acc + bias[n])
  kEpiBiasBf16 = 2,    // out bf16 = acc + bias[n]
  kEpiDgradElu = 3,    // out bf16 = acc * elu'(aux[m, n]) with aux = elu output (bf16); colsum partials of out
  kEpiPartialF32 = 4,  // out fp32 split partial: out[z * split_stride + m * ldo + n] = acc over split z
};

struct GemmParams {
  const void* a = nullptr;
  int lda = 0;
  bool a_mn_major = false;
  const void* b = nullptr;
  int ldb = 0;
  bool b_mn_major = false;
  int M = 0, N = 0, K = 0;
  int splits = 1;  // split-K over blockIdx.z (kEpiPartialF32 only)
  int epilogue = kEpiF32;
  void* out = nullptr;
  int ldo = 0;
  long long split_stride = 0;
  const float* bias = nullptr;
  const void* aux = nullptr;  // bf16 [M, ld_aux]
  int ld_aux = 0;
  float* colsum = nullptr;    // fp32 [colsum_rows, N]: per-CTA column sums of the stored output (bias gradients)
  int colsum_rows = 0;        // rows of colsum (>= the launch's CTA count, gemm_colsum_rows()); N <= kColsumMaxN
  unsigned int* status = nullptr;
};

// Widest output whose column sums the data-gradient epilogue accumulates per CTA (shared memory, fp32).
constexpr int kColsumMaxN = 1024;

// Returns cudaSuccess or the launch error. Host-side validation failures return cudaErrorInvalidValue.
cudaError_t gemm_launch(const GemmParams& p, cudaStream_t stream);

// Number of 128-row M tiles used for a given M.
inline int gemm_m_tiles(int M) { return (M + 127) / 128; }

// Rows of a column-sum partial buffer: one per CTA of the largest data-gradient launch (two CTAs per SM).
inline int gemm_colsum_rows(int sm_count) { return 2 * sm_count; }

}  // namespace rlb
