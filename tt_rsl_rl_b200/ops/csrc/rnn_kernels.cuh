// GRU / LSTM cell kernels of the fused recurrent PPO path (torch.nn.GRU / torch.nn.LSTM gate conventions).
//
// The gate pre-activations come from two tcgen05 GEMMs per step: gi = x W_ih^T + b_ih (all time steps of a minibatch
// at once) and gh = h W_hh^T + b_hh (one step at a time). The cells combine them:
//   GRU  (gates r, z, n): r = s(gi_r + gh_r), z = s(gi_z + gh_z), n = tanh(gi_n + r * gh_n), h' = (1 - z) n + z h
//   LSTM (gates i, f, g, o): i, f, o = s(gi + gh), g = tanh(gi_g + gh_g), c' = f c + i g, h' = o tanh(c')
// Episode boundaries are done-masks: the next step's input state is h' (1 - done) (and c' (1 - done)).
// Strides are in elements; every row-pitched array may be a strided view (env-major [env, T, width] buffers).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rlb {

struct RnnCellFwdArgs {
  int rows, H, lstm;
  const float* gi;  // [rows, G*H] (G = 3 GRU, 4 LSTM)
  long long ld_gi;
  const float* gh;
  long long ld_gh;
  const float* h_in;  // fp32 state entering the step
  long long ld_h_in;
  const float* c_in;  // LSTM cell state entering the step
  long long ld_c_in;
  float* h_out;  // optional fp32 h' (may alias h_in)
  long long ld_h_out;
  void* h_out_bf16;  // optional bf16 h' (GEMM operand of the head / next step)
  long long ld_h_out_bf16;
  float* c_out;  // LSTM c' (may alias c_in)
  long long ld_c_out;
  const float* done;  // optional [rows] done flags of this step: the next-step outputs below are masked by 1 - done
  float* next_h;      // optional fp32 h' (1 - done)
  long long ld_next_h;
  void* next_h_bf16;  // optional bf16 h' (1 - done)
  long long ld_next_h_bf16;
  float* next_c;  // LSTM: optional c' (1 - done)
  long long ld_next_c;
  float* save;  // optional saved activations [rows, S*H]: GRU r, z, n, gh_n (S = 4); LSTM i, f, g, o, tanh(c') (S = 5)
  long long ld_save;
};

struct RnnCellBwdArgs {
  int rows, H, lstm;
  const float* save;
  long long ld_save;
  const float* h_in;  // GRU: the step's input state (masked previous output)
  long long ld_h_in;
  const float* c_in;  // LSTM: the step's input cell state
  long long ld_c_in;
  // gradient reaching h' of this step: dh_head + (dh_rec_a + dh_rec_b) (1 - done), the recurrent part coming from the
  // next step's input state (which was h' (1 - done)); LSTM adds dc_rec (1 - done) to the cell-state gradient.
  const float* dh_head;
  long long ld_dh_head;
  const float* dh_rec_a;  // optional (null on the last step)
  const float* dh_rec_b;  // optional
  long long ld_dh_rec;
  const float* dc_rec;  // LSTM, optional
  long long ld_dc_rec;
  const float* done;  // optional [rows]
  // outputs
  void* dgi;  // bf16 [rows, G*H]: gradient of the input-side pre-activations
  long long ld_dgi;
  void* dgh;  // bf16 [rows, G*H] hidden-side (GRU only: differs in the n gate); null for LSTM (equal to dgi)
  long long ld_dgh;
  float* dh_direct;  // GRU: dL/dh_in not through W_hh (dh * z); null for LSTM
  long long ld_dh_direct;
  float* dc_prev;  // LSTM: dL/dc_in
  long long ld_dc_prev;
  float* colsum_gi;  // [blocks, G*H] per-block column sums of dgi (bias gradient of b_ih), optional
  float* colsum_gh;  // [blocks, G*H] of dgh (GRU), optional
  int colsum_accumulate;  // 1: add to the column sums (later steps of a BPTT sweep), 0: overwrite
};

// Rows handled by one block of the backward cell (the row count of its column-sum partials is ceil(rows / this)).
constexpr int kRnnBwdRows = 4;
inline int rnn_bwd_blocks(int rows) { return (rows + kRnnBwdRows - 1) / kRnnBwdRows; }

// dst = src (1 - done) for the fp32 state (and bf16 copy, and LSTM cell state); src may alias dst.
struct RnnMaskArgs {
  int rows, H;
  const float* src_h;
  long long ld_src_h;
  const float* src_c;
  long long ld_src_c;
  const float* done;  // optional
  float* dst_h;
  long long ld_dst_h;
  void* dst_h_bf16;
  long long ld_dst_h_bf16;
  float* dst_c;
  long long ld_dst_c;
};

// Zero-padded trajectory entries of a recurrent minibatch (environments lo .. lo + Be - 1 of a time-major done
// array [T, N]): every environment contributes one trajectory plus one per done before its last step, and each
// trajectory is padded to T steps, so out[0] = T * (number of nonzero done[t, e], t < T - 1). One block.
cudaError_t rnn_pad_entries(const float* done, int T, int N, int lo, int Be, float* out, cudaStream_t s);

cudaError_t rnn_cell_fwd(const RnnCellFwdArgs& a, cudaStream_t s);
cudaError_t rnn_cell_bwd(const RnnCellBwdArgs& a, cudaStream_t s);
cudaError_t rnn_mask(const RnnMaskArgs& a, cudaStream_t s);

}  // namespace rlb
