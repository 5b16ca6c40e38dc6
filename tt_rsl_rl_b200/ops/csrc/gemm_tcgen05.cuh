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
  kEpiRnnCell = 5,     // one GRU / LSTM step: the cell applied to gh = acc + bias (RnnCellEpi), no `out`
};

// Fused recurrent step (kEpiRnnCell): A = the bf16 input state [M, H] (K-major), B = W_hh [G*H, H] (K-major, G = 3
// GRU, 4 LSTM), N = G*H, K = H, bias = b_hh. A tile spans kRnnUnits hidden units of every gate (B rows g*H + u0 ..
// g*H + u0 + kRnnUnits - 1 for g = 0 .. G-1, loaded as G boxes), so its epilogue owns whole units and applies the
// torch.nn.GRU / torch.nn.LSTM cell with the gate order and outputs of rnn_kernels.cuh RnnCellFwdArgs. H must be a
// multiple of kRnnUnits; fp32 arrays need 16-byte aligned bases and pitches that are multiples of 4 elements, bf16
// arrays 16-byte aligned bases and pitches that are multiples of 8. No output may alias the A operand.
constexpr int kRnnUnits = 64;
struct RnnCellEpi {
  int H = 0, lstm = 0;
  const float* gi = nullptr;  // [M, G*H] input-side pre-activations (x W_ih^T + b_ih)
  long long ld_gi = 0;
  const float* h_in = nullptr;  // fp32 state entering the step
  long long ld_h_in = 0;
  const float* c_in = nullptr;  // LSTM cell state entering the step
  long long ld_c_in = 0;
  float* h_out = nullptr;  // optional fp32 h'
  long long ld_h_out = 0;
  void* h_out_bf16 = nullptr;  // optional bf16 h'
  long long ld_h_out_bf16 = 0;
  float* c_out = nullptr;  // optional LSTM c'
  long long ld_c_out = 0;
  const float* done = nullptr;  // optional [M]: the next-step outputs are masked by 1 - done
  float* next_h = nullptr;
  long long ld_next_h = 0;
  void* next_h_bf16 = nullptr;
  long long ld_next_h_bf16 = 0;
  float* next_c = nullptr;
  long long ld_next_c = 0;
  float* save = nullptr;  // optional [M, S*H]: GRU r, z, n, gh_n (S = 4); LSTM i, f, g, o, tanh(c') (S = 5)
  long long ld_save = 0;
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
  // kEpiF32: columns of each output row the epilogue may write (N .. ldo; 0 = N). Above N it stores whole 32-column
  // chunks (the padding columns receive zeros), so a padded output leaves through 16-byte row stores.
  int out_cols = 0;
  RnnCellEpi cell;            // kEpiRnnCell only
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
