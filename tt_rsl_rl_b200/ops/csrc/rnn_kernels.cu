// GRU / LSTM cells of the fused recurrent path (forward step, backward step with bias-gradient column sums, state
// masking). The recurrences of torch.nn.GRU / torch.nn.LSTM (rsl_rl/modules/rnn.py wraps them) in fp32.
#include <cuda_bf16.h>

#include "rnn_kernels.cuh"
#include "sm100_primitives.cuh"

namespace rlb {
namespace {

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + __expf(-x)); }

__device__ __forceinline__ void store_bf16(void* base, long long ld, int row, int col, float v) {
  static_cast<__nv_bfloat16*>(base)[static_cast<long long>(row) * ld + col] = __float2bfloat16_rn(v);
}

// one thread per (row, hidden unit)
__global__ void __launch_bounds__(256) rnn_cell_fwd_kernel(const RnnCellFwdArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const long long total = static_cast<long long>(a.rows) * a.H;
  const int H = a.H;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(e / H);
    const int j = static_cast<int>(e - static_cast<long long>(row) * H);
    const float* gi = a.gi + row * a.ld_gi;
    const float* gh = a.gh + row * a.ld_gh;
    // inputs are never written by this launch (outputs may alias h_in only element for element): non-coherent
    // loads, which the compiler may issue ahead of the previous element's stores
    const float h = __ldg(a.h_in + row * a.ld_h_in + j);
    float hn, cn = 0.f;
    if (!a.lstm) {
      const float r = sigmoid_f(__ldg(gi + j) + __ldg(gh + j));
      const float z = sigmoid_f(__ldg(gi + H + j) + __ldg(gh + H + j));
      const float ghn = __ldg(gh + 2 * H + j);
      const float n = tanhf(__ldg(gi + 2 * H + j) + r * ghn);
      hn = (1.0f - z) * n + z * h;
      if (a.save) {
        float* sv = a.save + row * a.ld_save;
        sv[j] = r;
        sv[H + j] = z;
        sv[2 * H + j] = n;
        sv[3 * H + j] = ghn;
      }
    } else {
      const float c = __ldg(a.c_in + row * a.ld_c_in + j);
      const float ig = sigmoid_f(__ldg(gi + j) + __ldg(gh + j));
      const float fg = sigmoid_f(__ldg(gi + H + j) + __ldg(gh + H + j));
      const float gg = tanhf(__ldg(gi + 2 * H + j) + __ldg(gh + 2 * H + j));
      const float og = sigmoid_f(__ldg(gi + 3 * H + j) + __ldg(gh + 3 * H + j));
      cn = fg * c + ig * gg;
      const float tc = tanhf(cn);
      hn = og * tc;
      if (a.save) {
        float* sv = a.save + row * a.ld_save;
        sv[j] = ig;
        sv[H + j] = fg;
        sv[2 * H + j] = gg;
        sv[3 * H + j] = og;
        sv[4 * H + j] = tc;
      }
      if (a.c_out) a.c_out[row * a.ld_c_out + j] = cn;
    }
    if (a.h_out) a.h_out[row * a.ld_h_out + j] = hn;
    if (a.h_out_bf16) store_bf16(a.h_out_bf16, a.ld_h_out_bf16, row, j, hn);
    const float keep = a.done ? 1.0f - __ldg(a.done + row) : 1.0f;
    if (a.next_h) a.next_h[row * a.ld_next_h + j] = hn * keep;
    if (a.next_h_bf16) store_bf16(a.next_h_bf16, a.ld_next_h_bf16, row, j, hn * keep);
    if (a.lstm && a.next_c) a.next_c[row * a.ld_next_c + j] = cn * keep;
  }
}

constexpr int kBwdThreads = 256;
constexpr int kMaxColIter = 4;  // H <= 1024

// A block takes kRnnBwdRows rows; thread t handles hidden units t, t + 256, ... of every row and keeps the column
// sums of its gate gradients in registers (written once per block: deterministic partials).
// KI = ceil(H / 256) unit slots per thread (a kernel per KI: the column-sum registers of unused slots would cost
// occupancy; H = 256 runs KI = 1).
template <int KI>
__global__ void __launch_bounds__(kBwdThreads) rnn_cell_bwd_kernel(const RnnCellBwdArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const int H = a.H;
  const int G = a.lstm ? 4 : 3;
  const int row0 = blockIdx.x * kRnnBwdRows;
  float cs_gi[4][KI];
  float cs_ghn[KI];
#pragma unroll
  for (int k = 0; k < KI; ++k) {
    cs_ghn[k] = 0.f;
#pragma unroll
    for (int g = 0; g < 4; ++g) cs_gi[g][k] = 0.f;
  }
  for (int rr = 0; rr < kRnnBwdRows; ++rr) {
    const int row = row0 + rr;
    if (row >= a.rows) break;
    const float keep = a.done ? 1.0f - a.done[row] : 1.0f;
    const float* sv = a.save + row * a.ld_save;
#pragma unroll
    for (int k = 0; k < KI; ++k) {
      const int j = threadIdx.x + k * kBwdThreads;
      if (j >= H) break;
      float dh = a.dh_head[row * a.ld_dh_head + j];
      float rec = 0.f;
      if (a.dh_rec_a) rec += a.dh_rec_a[row * a.ld_dh_rec + j];
      if (a.dh_rec_b) rec += a.dh_rec_b[row * a.ld_dh_rec + j];
      dh += rec * keep;
      if (!a.lstm) {
        const float r = sv[j], z = sv[H + j], n = sv[2 * H + j], ghn = sv[3 * H + j];
        const float h = a.h_in[row * a.ld_h_in + j];
        const float dn = dh * (1.0f - z);
        const float dz = dh * (h - n);
        const float da_n = dn * (1.0f - n * n);
        const float da_r = da_n * ghn * r * (1.0f - r);
        const float da_z = dz * z * (1.0f - z);
        const float dgh_n = da_n * r;
        store_bf16(a.dgi, a.ld_dgi, row, j, da_r);
        store_bf16(a.dgi, a.ld_dgi, row, H + j, da_z);
        store_bf16(a.dgi, a.ld_dgi, row, 2 * H + j, da_n);
        store_bf16(a.dgh, a.ld_dgh, row, j, da_r);
        store_bf16(a.dgh, a.ld_dgh, row, H + j, da_z);
        store_bf16(a.dgh, a.ld_dgh, row, 2 * H + j, dgh_n);
        if (a.dh_direct) a.dh_direct[row * a.ld_dh_direct + j] = dh * z;
        cs_gi[0][k] += da_r;
        cs_gi[1][k] += da_z;
        cs_gi[2][k] += da_n;
        cs_ghn[k] += dgh_n;
      } else {
        const float ig = sv[j], fg = sv[H + j], gg = sv[2 * H + j], og = sv[3 * H + j], tc = sv[4 * H + j];
        const float c = a.c_in[row * a.ld_c_in + j];
        float dc = dh * og * (1.0f - tc * tc);
        if (a.dc_rec) dc += a.dc_rec[row * a.ld_dc_rec + j] * keep;
        const float da_i = dc * gg * ig * (1.0f - ig);
        const float da_f = dc * c * fg * (1.0f - fg);
        const float da_g = dc * ig * (1.0f - gg * gg);
        const float da_o = dh * tc * og * (1.0f - og);
        store_bf16(a.dgi, a.ld_dgi, row, j, da_i);
        store_bf16(a.dgi, a.ld_dgi, row, H + j, da_f);
        store_bf16(a.dgi, a.ld_dgi, row, 2 * H + j, da_g);
        store_bf16(a.dgi, a.ld_dgi, row, 3 * H + j, da_o);
        if (a.dc_prev) a.dc_prev[row * a.ld_dc_prev + j] = dc * fg;
        cs_gi[0][k] += da_i;
        cs_gi[1][k] += da_f;
        cs_gi[2][k] += da_g;
        cs_gi[3][k] += da_o;
      }
    }
  }
  const long long GH = static_cast<long long>(G) * H;
#pragma unroll
  for (int k = 0; k < KI; ++k) {
    const int j = threadIdx.x + k * kBwdThreads;
    if (j >= H) break;
    // one partial row per block, accumulated over the steps of a BPTT sweep (steps run in stream order)
    auto put = [&](float* o, float v) { *o = a.colsum_accumulate ? *o + v : v; };
    if (a.colsum_gi) {
      float* o = a.colsum_gi + blockIdx.x * GH;
      for (int g = 0; g < G; ++g) put(o + g * H + j, cs_gi[g][k]);
    }
    if (a.colsum_gh) {
      float* o = a.colsum_gh + blockIdx.x * GH;
      put(o + j, cs_gi[0][k]);
      put(o + H + j, cs_gi[1][k]);
      put(o + 2 * H + j, a.lstm ? cs_gi[2][k] : cs_ghn[k]);
      if (a.lstm) put(o + 3 * H + j, cs_gi[3][k]);
    }
  }
}

__global__ void __launch_bounds__(256) rnn_mask_kernel(const RnnMaskArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const long long total = static_cast<long long>(a.rows) * a.H;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(e / a.H);
    const int j = static_cast<int>(e - static_cast<long long>(row) * a.H);
    const float keep = a.done ? 1.0f - a.done[row] : 1.0f;
    const float h = a.src_h[row * a.ld_src_h + j] * keep;
    if (a.dst_h) a.dst_h[row * a.ld_dst_h + j] = h;
    if (a.dst_h_bf16) store_bf16(a.dst_h_bf16, a.ld_dst_h_bf16, row, j, h);
    if (a.src_c && a.dst_c) a.dst_c[row * a.ld_dst_c + j] = a.src_c[row * a.ld_src_c + j] * keep;
  }
}

// One block of 256 threads: integer counts per thread, a warp butterfly and a fixed-order sum of the eight warps
// (exact, so the result is independent of the launch shape).
__global__ void __launch_bounds__(256) rnn_pad_entries_kernel(const float* done, int T, int N, int lo, int Be,
                                                              float* out) {
  const long long n = static_cast<long long>(T - 1) * Be;
  int count = 0;
  for (long long k = threadIdx.x; k < n; k += blockDim.x) {
    const int t = static_cast<int>(k / Be);
    const int e = static_cast<int>(k - static_cast<long long>(t) * Be);
    count += done[static_cast<long long>(t) * N + lo + e] != 0.0f ? 1 : 0;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) count += __shfl_xor_sync(0xffffffffu, count, off);
  __shared__ int s_count[8];
  if ((threadIdx.x & 31) == 0) s_count[threadIdx.x >> 5] = count;
  __syncthreads();
  if (threadIdx.x == 0) {
    long long total = 0;
    for (int w = 0; w < 8; ++w) total += s_count[w];
    out[0] = static_cast<float>(total * T);
  }
}

int elementwise_grid(long long n) {
  long long blocks = (n + 255) / 256;
  const long long cap = 148LL * 32;  // one element per thread up to ~1.2 M elements (a minibatch step)
  return static_cast<int>(blocks < cap ? (blocks < 1 ? 1 : blocks) : cap);
}

}  // namespace

cudaError_t rnn_pad_entries(const float* done, int T, int N, int lo, int Be, float* out, cudaStream_t s) {
  if (!done || !out || T <= 0 || Be <= 0 || lo < 0 || lo + Be > N) return cudaErrorInvalidValue;
  rnn_pad_entries_kernel<<<1, 256, 0, s>>>(done, T, N, lo, Be, out);
  return cudaGetLastError();
}

cudaError_t rnn_cell_fwd(const RnnCellFwdArgs& a, cudaStream_t s) {
  if (a.rows <= 0 || a.H <= 0 || !a.gi || !a.gh || !a.h_in || (a.lstm && !a.c_in)) return cudaErrorInvalidValue;
  launch_pdl(rnn_cell_fwd_kernel, dim3(elementwise_grid(static_cast<long long>(a.rows) * a.H)), dim3(256), 0, s, a);
  return cudaGetLastError();
}

cudaError_t rnn_cell_bwd(const RnnCellBwdArgs& a, cudaStream_t s) {
  if (a.rows <= 0 || a.H <= 0 || a.H > kBwdThreads * kMaxColIter || !a.save || !a.dh_head || !a.dgi)
    return cudaErrorInvalidValue;
  if (!a.lstm && (!a.h_in || !a.dgh)) return cudaErrorInvalidValue;
  if (a.lstm && !a.c_in) return cudaErrorInvalidValue;
  const int ki = (a.H + kBwdThreads - 1) / kBwdThreads;
  const int blocks = rnn_bwd_blocks(a.rows);
  if (ki == 1) launch_pdl(rnn_cell_bwd_kernel<1>, dim3(blocks), dim3(kBwdThreads), 0, s, a);
  else if (ki == 2) launch_pdl(rnn_cell_bwd_kernel<2>, dim3(blocks), dim3(kBwdThreads), 0, s, a);
  else launch_pdl(rnn_cell_bwd_kernel<4>, dim3(blocks), dim3(kBwdThreads), 0, s, a);
  return cudaGetLastError();
}

cudaError_t rnn_mask(const RnnMaskArgs& a, cudaStream_t s) {
  if (a.rows <= 0 || a.H <= 0 || !a.src_h) return cudaErrorInvalidValue;
  launch_pdl(rnn_mask_kernel, dim3(elementwise_grid(static_cast<long long>(a.rows) * a.H)), dim3(256), 0, s, a);
  return cudaGetLastError();
}

}  // namespace rlb
