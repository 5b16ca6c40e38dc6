// RL kernels for sm_100a: rollout head, environment-step bookkeeping, GAE, minibatch gather, PPO loss, gradient
// reduction, fused clip + Adam (with the peer-to-peer data-parallel exchange) and the observation normaliser.
//
// Determinism: every cross-thread reduction runs in a fixed order (per-block partials, then a fixed-order sum), so a
// replay of the same inputs is bit-identical and every data-parallel rank computes identical parameters.
#include <cuda_bf16.h>

#include <cmath>
#include <cstdio>

#include "philox.cuh"
#include "rl_kernels.cuh"
#include "sm100_primitives.cuh"

namespace rlb {
namespace {

constexpr float kLogSqrt2Pi = 0.91893853320467274178f;  // 0.5 * ln(2 * pi)

__device__ __forceinline__ float load_flag(const void* p, int dtype, int i) {
  if (dtype == 0) return static_cast<const float*>(p)[i] != 0.f ? 1.f : 0.f;
  if (dtype == 1) return static_cast<const uint8_t*>(p)[i] != 0 ? 1.f : 0.f;
  return static_cast<const long long*>(p)[i] != 0 ? 1.f : 0.f;
}

// ---------------------------------------------------------------------------------------------------------------
// prep_obs
// ---------------------------------------------------------------------------------------------------------------
constexpr int kPrepMaxD = 1024;
// One warp per row; lanes walk the columns of each group (coalesced), normaliser constants staged in shared memory.
__global__ void __launch_bounds__(256) prep_obs_kernel(const PrepObsArgs a, int D) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  __shared__ float s_mean[kPrepMaxD];
  __shared__ float s_inv[kPrepMaxD];
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    s_mean[c] = a.mean ? a.mean[c] : 0.f;
    s_inv[c] = a.mean ? 1.0f / (a.std[c] + a.eps) : 1.f;
  }
  __syncthreads();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  __nv_bfloat16* x = static_cast<__nv_bfloat16*>(a.x);
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < a.rows; r += gridDim.x * warps) {
    int base = 0;
    for (int g = 0; g < a.groups; ++g) {
      const float* src = a.src[g] + static_cast<size_t>(r) * a.src_ld[g];
      for (int c = lane; c < a.width[g]; c += 32) {
        const float v = src[c];
        const int col = base + c;
        if (a.store) a.store[static_cast<size_t>(r) * a.ld_store + col] = v;
        x[static_cast<size_t>(r) * a.ld_x + col] = __float2bfloat16_rn((v - s_mean[col]) * s_inv[col]);
      }
      base += a.width[g];
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Gaussian head (rollout): one warp per row, lane j handles actions j, j + 32, ...
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float head_std(float raw, int log_std, float lo, float hi, float llo, float lhi) {
  return log_std ? expf(fminf(fmaxf(raw, llo), lhi)) : fminf(fmaxf(raw, lo), hi);
}

// After every block has read the counter, the last block to finish advances it (ticket pattern).
__device__ __forceinline__ void last_block_advance(uint64_t* counter, unsigned int* ticket) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int done = atomicAdd(ticket, 1u) + 1u;
    if (done == gridDim.x) {
      *counter += 1;
      *ticket = 0u;
      __threadfence();
    }
  }
}

__global__ void gaussian_sample_kernel(const SampleArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t offset = *a.counter;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < a.rows; row += gridDim.x * warps) {
    float logp = 0.f;
    for (int j0 = 0; j0 < a.A; j0 += 32) {
      const int j = j0 + lane;
      // 4 normals per Philox call: counter = (row, action-group of 4, offset lo, offset hi)
      const int grp = j >> 2;
      const Philox rnd = philox10(static_cast<uint32_t>(row), static_cast<uint32_t>(grp),
                                  static_cast<uint32_t>(offset), static_cast<uint32_t>(offset >> 32),
                                  static_cast<uint32_t>(a.seed), static_cast<uint32_t>(a.seed >> 32));
      float n0, n1, n2, n3;
      box_muller(rnd.c[0], rnd.c[1], n0, n1);
      box_muller(rnd.c[2], rnd.c[3], n2, n3);
      const int k = j & 3;
      const float eps = k == 0 ? n0 : k == 1 ? n1 : k == 2 ? n2 : n3;
      if (j < a.A) {
        const float* h = a.head + static_cast<size_t>(row) * a.ld_head;
        const float mu = h[j];
        const float raw = a.hetero ? h[a.A + j] : a.std_param[j];
        const float sd = head_std(raw, a.log_std, a.std_lo, a.std_hi, a.log_std_lo, a.log_std_hi);
        const float act = mu + sd * eps;
        const size_t o = static_cast<size_t>(row) * a.A + j;
        a.actions[o] = act;
        if (a.actions_copy) a.actions_copy[o] = act;
        a.out_mean[o] = mu;
        a.out_std[o] = sd;
        const float z = (act - mu) / sd;
        logp += -0.5f * z * z - logf(sd) - kLogSqrt2Pi;
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) logp += __shfl_xor_sync(0xffffffffu, logp, off);
    if (lane == 0) a.out_logp[row] = logp;
  }
  last_block_advance(a.counter, a.ticket);
}

// A <= 32: eight lanes per row, four rows per warp. Lane l8 of a row owns actions 4 l8 .. 4 l8 + 3, which are exactly
// the four normals of one Philox block (counter word 1 = action group), so each block is computed once instead of by
// four lanes; same streams and results as gaussian_sample_kernel.
__global__ void __launch_bounds__(256) gaussian_sample_rows8_kernel(const SampleArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int l8 = lane & 7;
  const uint64_t offset = *a.counter;
  const int rows_per_block = (blockDim.x >> 5) * 4;
  for (int row0 = blockIdx.x * rows_per_block; row0 < a.rows; row0 += gridDim.x * rows_per_block) {
    const int row = row0 + (threadIdx.x >> 5) * 4 + (lane >> 3);
    const bool in = row < a.rows;
    float logp = 0.f;
    if (in && 4 * l8 < a.A) {
      const Philox rnd = philox10(static_cast<uint32_t>(row), static_cast<uint32_t>(l8),
                                  static_cast<uint32_t>(offset), static_cast<uint32_t>(offset >> 32),
                                  static_cast<uint32_t>(a.seed), static_cast<uint32_t>(a.seed >> 32));
      float eps[4];
      box_muller(rnd.c[0], rnd.c[1], eps[0], eps[1]);
      box_muller(rnd.c[2], rnd.c[3], eps[2], eps[3]);
      const float* h = a.head + static_cast<size_t>(row) * a.ld_head;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = 4 * l8 + k;
        if (j < a.A) {
          const float mu = h[j];
          const float raw = a.hetero ? h[a.A + j] : a.std_param[j];
          const float sd = head_std(raw, a.log_std, a.std_lo, a.std_hi, a.log_std_lo, a.log_std_hi);
          const float act = mu + sd * eps[k];
          const size_t o = static_cast<size_t>(row) * a.A + j;
          a.actions[o] = act;
          if (a.actions_copy) a.actions_copy[o] = act;
          a.out_mean[o] = mu;
          a.out_std[o] = sd;
          const float z = (act - mu) / sd;
          logp += -0.5f * z * z - logf(sd) - kLogSqrt2Pi;
        }
      }
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) logp += __shfl_xor_sync(0xffffffffu, logp, off);
    if (in && l8 == 0) a.out_logp[row] = logp;
  }
  last_block_advance(a.counter, a.ticket);
}

// ---------------------------------------------------------------------------------------------------------------
// process_step
// ---------------------------------------------------------------------------------------------------------------
__global__ void process_step_kernel(const ProcessArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.rows; i += gridDim.x * blockDim.x) {
    float r = a.rewards[i];
    if (a.intrinsic) r += a.intrinsic[i];
    if (a.timeouts) r += a.gamma * a.values_slot[i] * load_flag(a.timeouts, a.timeouts_dtype, i);
    if (a.nonfinite_flag && !isfinite(r)) atomicExch(a.nonfinite_flag, 1u);
    a.rewards_slot[i] = r;
    a.dones_slot[i] = load_flag(a.dones, a.dones_dtype, i);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// GAE: one thread per environment, reverse scan over T
// ---------------------------------------------------------------------------------------------------------------
constexpr int kGaeThreads = 256;
__global__ void gae_kernel(const GaeArgs a) {
  const int n = blockIdx.x * kGaeThreads + threadIdx.x;
  double s = 0.0, ss = 0.0;
  if (n < a.N) {
    float adv = 0.f;
    float next_v = a.last_values[n];
    for (int t = a.T - 1; t >= 0; --t) {
      const size_t o = static_cast<size_t>(t) * a.N + n;
      const float v = a.values[o];
      const float not_done = 1.0f - a.dones[o];
      const float delta = a.rewards[o] + not_done * a.gamma * next_v - v;
      adv = delta + not_done * a.gamma * a.lam * adv;
      const float ret = adv + v;
      a.returns[o] = ret;
      const float ad = ret - v;  // advantages = returns - values (as stored upstream)
      a.advantages[o] = ad;
      s += ad;
      ss += static_cast<double>(ad) * ad;
      next_v = v;
    }
  }
  __shared__ double sh[2][kGaeThreads / 32];
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, off);
    ss += __shfl_xor_sync(0xffffffffu, ss, off);
  }
  if ((threadIdx.x & 31) == 0) {
    sh[0][threadIdx.x >> 5] = s;
    sh[1][threadIdx.x >> 5] = ss;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0, tss = 0;
    for (int w = 0; w < kGaeThreads / 32; ++w) {
      ts += sh[0][w];
      tss += sh[1][w];
    }
    a.partial[2 * blockIdx.x] = ts;
    a.partial[2 * blockIdx.x + 1] = tss;
  }
}

__global__ void adv_normalize_kernel(float* adv, long long n, const double* partial, int parts) {
  __shared__ float stats[2];
  __shared__ double red[2][32];
  // every block reduces the per-block GAE partials in the same fixed tree order
  double s = 0.0, ss = 0.0;
  for (int i = threadIdx.x; i < parts; i += blockDim.x) {
    s += partial[2 * i];
    ss += partial[2 * i + 1];
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, off);
    ss += __shfl_xor_sync(0xffffffffu, ss, off);
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = s;
    red[1][threadIdx.x >> 5] = ss;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0, tss = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
      ts += red[0][w];
      tss += red[1][w];
    }
    const double mean = ts / static_cast<double>(n);
    const double var = n > 1 ? fmax((tss - ts * mean) / static_cast<double>(n - 1), 0.0) : 0.0;
    stats[0] = static_cast<float>(mean);
    stats[1] = static_cast<float>(1.0 / (sqrt(var) + 1e-8));
  }
  __syncthreads();
  const float mean = stats[0], inv = stats[1];
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    adv[i] = (adv[i] - mean) * inv;
}

constexpr int kAdvGatherBlocks = 148;

__global__ void __launch_bounds__(256) adv_gather_stats_kernel(const float* __restrict__ adv, long long n_adv,
                                                                const int* __restrict__ idx, long long n,
                                                                float* __restrict__ out, double* __restrict__ partial,
                                                                unsigned int* status) {
  __shared__ double red[2][8];
  double s = 0.0, ss = 0.0;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    long long src = idx[i];
    RL_CHECK_INDEX(src, n_adv, status, 43);
    const float v = adv[src];
    out[i] = v;
    s += v;
    ss += static_cast<double>(v) * v;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, off);
    ss += __shfl_xor_sync(0xffffffffu, ss, off);
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = s;
    red[1][threadIdx.x >> 5] = ss;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0, tss = 0;
    for (int w = 0; w < 8; ++w) {
      ts += red[0][w];
      tss += red[1][w];
    }
    partial[2 * blockIdx.x] = ts;
    partial[2 * blockIdx.x + 1] = tss;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Feistel permutation of [0, n): 4-round balanced Feistel network on 2*half_bits bits with cycle walking. A bijection
// of the padded domain restricted by cycle walking is a bijection of [0, n).
// ---------------------------------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t mix32(uint32_t x, uint32_t key, uint32_t round) {
  uint32_t h = x * 0x9E3779B1u ^ (key + round * 0x85EBCA77u);
  h ^= h >> 15;
  h *= 0x2C1B3C6Du;
  h ^= h >> 12;
  h *= 0x297A2D39u;
  h ^= h >> 15;
  return h;
}
__host__ __device__ __forceinline__ uint32_t feistel_once(uint32_t x, uint32_t half_bits, uint32_t key) {
  const uint32_t mask = (1u << half_bits) - 1u;
  uint32_t L = x >> half_bits, R = x & mask;
  for (uint32_t r = 0; r < 4; ++r) {
    const uint32_t nl = R;
    R = L ^ (mix32(R, key, r) & mask);
    L = nl;
  }
  return (L << half_bits) | R;
}
__host__ __device__ __forceinline__ uint32_t feistel_permute(uint32_t i, uint32_t n, uint32_t half_bits, uint32_t key,
                                                             bool* overflow) {
  uint32_t x = feistel_once(i, half_bits, key);
  // Cycle walking terminates (the cycle through i < n returns to [0, n)); the cap only guards against misuse.
  for (int it = 0; x >= n; ++it) {
    if (it > (1 << 22)) {
      *overflow = true;
      return i;
    }
    x = feistel_once(x, half_bits, key);
  }
  return x;
}

constexpr int kGatherMaxD = 1024;
constexpr int kGatherRows = 8;  // rows per warp iteration (their loads are issued together)
// One warp gathers kGatherRows rows at a time: lanes 0..R-1 compute the permuted source rows (and symmetry copies),
// then lane l handles columns [4l, 4l + 4) of every row of the batch (128 columns per pass): a 16-byte load per row
// when the source row pitch allows it (identity copies), else four scalar loads through the copy's column map. All
// R rows' loads are issued before any conversion, so each warp keeps R 16-byte loads in flight.
// Source column of a mirrored copy (a host-probed signed permutation); checked in RL_DEBUG_BOUNDS builds (site 42).
__device__ __forceinline__ int perm_col(const int* p, int n, unsigned int* status) {
  int j = __ldg(p);
  RL_CHECK_INDEX(j, n, status, 42);
  return j;
}

__global__ void __launch_bounds__(256, 3) gather_minibatch_kernel(const GatherArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  __shared__ __align__(16) float s_mean[kGatherModels][kGatherMaxD];
  __shared__ __align__(16) float s_inv[kGatherModels][kGatherMaxD];
  int max_rows = 0;
  for (int m = 0; m < a.models; ++m) {
    max_rows = max(max_rows, a.rows[m]);
    for (int c = threadIdx.x; c < kGatherMaxD; c += blockDim.x) {
      const bool in = c < a.dim[m];
      s_mean[m][c] = (in && a.mean[m]) ? a.mean[m][c] : 0.f;
      s_inv[m][c] = (in && a.mean[m]) ? 1.0f / (a.std[m][c] + a.eps) : 1.f;
    }
  }
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t key = a.key_ptr ? *a.key_ptr : 0u;
  for (int i0 = (blockIdx.x * warps + (threadIdx.x >> 5)) * kGatherRows; i0 < max_rows;
       i0 += gridDim.x * warps * kGatherRows) {
    // row i is copy i / B of original sample i % B (computed once per row by lanes 0..R-1)
    int my_src = 0, my_copy = 0;
    if (lane < kGatherRows && i0 + lane < max_rows) {
      const int i = i0 + lane;
      my_copy = a.copies > 1 ? i / a.B : 0;
      const int o = i - my_copy * a.B;
      if (a.idx_in) {
        my_src = a.idx_in[o];
        RL_CHECK_INDEX(my_src, a.total, a.status, 41);
      } else {
        bool overflow = false;
        my_src = static_cast<int>(feistel_permute(static_cast<uint32_t>(a.offset + o), static_cast<uint32_t>(a.total),
                                                  a.half_bits, key, &overflow));
        if (overflow) report_error(a.status, kBadShape, 40);
      }
      if (a.idx_out && i < a.B) a.idx_out[i] = my_src;
    }
    int src[kGatherRows], cp[kGatherRows];
#pragma unroll
    for (int r = 0; r < kGatherRows; ++r) {
      src[r] = __shfl_sync(0xffffffffu, my_src, r);
      cp[r] = __shfl_sync(0xffffffffu, my_copy, r);
    }
    for (int m = 0; m < a.models; ++m) {
      const int D = a.dim[m];
      const int rows_m = a.rows[m];
      if (i0 >= rows_m) continue;
      const int* perm = a.perm[m];
      const float* sign = a.sign[m];
      const float* obs = a.obs[m];
      const int ld = a.obs_ld[m];
      const bool vec = a.vec4[m] != 0;
      for (int c = 4 * lane; c < D; c += 128) {
        float4 v[kGatherRows];
#pragma unroll
        for (int r = 0; r < kGatherRows; ++r) {
          v[r] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (i0 + r < rows_m) {
            const float* row = obs + static_cast<size_t>(src[r]) * ld;
            if (perm != nullptr && cp[r] > 0) {  // mirrored copy: signed column permutation of the raw observation
              const int* pc = perm + cp[r] * D + c;
              const float* sc = sign + cp[r] * D + c;
              v[r].x = __ldg(sc) * __ldg(row + perm_col(pc, D, a.status));
              if (c + 1 < D) v[r].y = __ldg(sc + 1) * __ldg(row + perm_col(pc + 1, D, a.status));
              if (c + 2 < D) v[r].z = __ldg(sc + 2) * __ldg(row + perm_col(pc + 2, D, a.status));
              if (c + 3 < D) v[r].w = __ldg(sc + 3) * __ldg(row + perm_col(pc + 3, D, a.status));
            } else if (vec) {  // the row pitch is a multiple of 4 floats: columns past D are in-row padding
              v[r] = __ldg(reinterpret_cast<const float4*>(row + c));
            } else {
              v[r].x = __ldg(row + c);
              if (c + 1 < D) v[r].y = __ldg(row + c + 1);
              if (c + 2 < D) v[r].z = __ldg(row + c + 2);
              if (c + 3 < D) v[r].w = __ldg(row + c + 3);
            }
          }
        }
        const float4 mu = *reinterpret_cast<const float4*>(&s_mean[m][c]);
        float4 inv = *reinterpret_cast<const float4*>(&s_inv[m][c]);
        // columns at or past D are written as zeros (the padding of the bf16 row)
        if (c + 1 >= D) inv.y = 0.f;
        if (c + 2 >= D) inv.z = 0.f;
        if (c + 3 >= D) inv.w = 0.f;
#pragma unroll
        for (int r = 0; r < kGatherRows; ++r) {
          if (i0 + r < rows_m) {
            uint2 w;
            w.x = pack_bf16x2((v[r].x - mu.x) * inv.x, (v[r].y - mu.y) * inv.y);
            w.y = pack_bf16x2((v[r].z - mu.z) * inv.z, (v[r].w - mu.w) * inv.w);
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.x[m]) + static_cast<size_t>(i0 + r) * a.ld_x[m] +
                                      c) = w;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// PPO loss: one warp per row (lane j handles actions j and j + 32); 16 warps x 4 rows per block
// ---------------------------------------------------------------------------------------------------------------
constexpr int kLossWarps = 8;
constexpr int kLossRowsPerWarp = 4;
constexpr int kLossRowsPerBlock = kLossWarps * kLossRowsPerWarp;
constexpr int kLossMaxA = 64;
constexpr int kLossGridCap = 2 * 148;  // two resident blocks per SM of a B200

// Standard deviation of the head's std parameterisation and its log and reciprocal: with log-std the log is the
// clamped raw value itself (no logarithm), with a direct std one log; one correctly rounded reciprocal replaces the
// divisions of the log-probability, KL and gradient terms.
__device__ __forceinline__ void std_terms(float raw, const PpoLossArgs& a, float& sd, float& lsd, float& isd) {
  if (a.log_std) {
    lsd = fminf(fmaxf(raw, a.log_std_lo), a.log_std_hi);
    sd = expf(lsd);
  } else {
    sd = fminf(fmaxf(raw, a.std_lo), a.std_hi);
    lsd = logf(sd);
  }
  isd = __frcp_rn(sd);
}

// torch.max(a, b) backward: the larger input gets the gradient, ties split it in halves.
__device__ __forceinline__ void max_grad_split(float a, float b, float& ga, float& gb) {
  ga = a > b ? 1.f : (a == b ? 0.5f : 0.f);
  gb = b > a ? 1.f : (a == b ? 0.5f : 0.f);
}

// Row i of the minibatch is symmetry copy i / n0 of original sample i % n0 (copy 0: the sample itself). Terms:
//   surrogate and value: rows of every copy with data augmentation (mean over B), else copy 0 (mean over n0);
//   entropy and KL: copy 0 only (mean over n0), as upstream evaluates them on the original samples;
//   mirror loss: copies >= 1, MSE between the row's mean and the mirrored mean of its original (target detached).
// kSym = false compiles the plain path (one copy) without the symmetry branches and their registers.
// Both paths first issue every load of the warp's kLossRowsPerWarp rows (random storage rows: actions, old mean and
// std, scalars; with copies the permuted actions and mirror targets) and only then compute, so each warp keeps its
// rows' loads in flight together.
template <bool kSym>
__global__ void __launch_bounds__(kLossWarps * 32, 2) ppo_loss_kernel(const PpoLossArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const float invP = 1.0f / static_cast<float>(a.aug ? a.B : a.n0);
  const float invE = 1.0f / static_cast<float>(a.n0);
  const float invM = a.copies > 1 ? 1.0f / (static_cast<float>(a.B - a.n0) * static_cast<float>(a.A)) : 0.f;
  const int head_cols = a.hetero ? 2 * a.A : a.A;
  // per-lane accumulators: columns lane and lane + 32 of the head gradient, std gradient
  float acc_dh[4] = {0.f, 0.f, 0.f, 0.f};  // head cols lane, lane+32, lane+64, lane+96
  float acc_dstd[2] = {0.f, 0.f};
  float acc_surr = 0.f, acc_val = 0.f, acc_ent = 0.f, acc_kl = 0.f, acc_sym = 0.f, acc_dv = 0.f;

  // state-independent std (a parameter): std, log std and 1 / std of this lane's actions, once per kernel
  float c_raw[2], c_sd[2], c_lsd[2], c_isd[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int j = lane + 32 * k;
    c_raw[k] = (!a.hetero && j < a.A) ? a.std_param[j] : 1.f;
    std_terms(c_raw[k], a, c_sd[k], c_lsd[k], c_isd[k]);
  }
  // blocks stride over groups of kLossRowsPerBlock rows: the grid (and so the number of per-block partials that the
  // gradient reduction has to sum) is capped at kLossGridCap whatever the minibatch size
  const int ngroups = (a.B + kLossRowsPerBlock - 1) / kLossRowsPerBlock;
  for (int grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
  const int row0 = grp * kLossRowsPerBlock + warp * kLossRowsPerWarp;
  // prefetch: every load of this warp's rows (random storage rows; with symmetry copies the signed-permuted action
  // columns and the mirror targets) before any arithmetic
  constexpr int PF = kLossRowsPerWarp;
  float pf_act[PF][2], pf_omu[PF][2], pf_osd[PF][2], pf_mu[PF][2], pf_raw[PF][2], pf_mt[PF][2];
  float pf_adv[PF], pf_lp[PF], pf_ret[PF], pf_vold[PF], pf_v[PF];
#pragma unroll
  for (int rr = 0; rr < PF; ++rr) {
    const int i = row0 + rr;
    const bool in = i < a.B;
    const int copy = (kSym && in) ? i / a.n0 : 0;
    const int o = in ? i - copy * a.n0 : 0;
    int src = in ? a.idx[o] : 0;
    RL_CHECK_INDEX(src, a.total, a.status, 44);
    const float* h = a.head + static_cast<size_t>(in ? i : 0) * a.ld_head;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int j = lane + 32 * k;
      const bool ok = in && j < a.A;
      int aj = j;
      float asg = 1.f, mt = 0.f;
      if (kSym && ok && copy > 0) {  // the copy's action and mirror target: signed permutation of the original's
        aj = a.act_perm[copy * a.A + j];
        RL_CHECK_INDEX(aj, a.A, a.status, 45);
        asg = a.act_sign[copy * a.A + j];
        mt = asg * a.head[static_cast<size_t>(o) * a.ld_head + aj];
      }
      const size_t so = static_cast<size_t>(src) * a.A + j;
      pf_act[rr][k] = ok ? asg * a.st_actions[static_cast<size_t>(src) * a.A + aj] : 0.f;
      pf_omu[rr][k] = (ok && copy == 0) ? a.st_mean[so] : 0.f;
      pf_osd[rr][k] = (ok && copy == 0) ? a.st_std[so] : 1.f;
      pf_mu[rr][k] = ok ? h[j] : 0.f;
      pf_raw[rr][k] = (ok && a.hetero) ? h[a.A + j] : 1.f;  // non-hetero: the shared parameter, read below
      pf_mt[rr][k] = mt;
    }
    pf_adv[rr] = in ? (a.adv_override ? a.adv_override[o] : a.st_adv[src]) : 0.f;
    pf_lp[rr] = in ? a.st_logp[src] : 0.f;
    pf_ret[rr] = in ? a.st_ret[src] : 0.f;
    pf_vold[rr] = in ? a.st_val[src] : 0.f;
    pf_v[rr] = in ? a.value[static_cast<size_t>(i) * a.ld_value] : 0.f;
  }
#pragma unroll
  for (int rr = 0; rr < kLossRowsPerWarp; ++rr) {
    const int i = row0 + rr;
    if (i >= a.B) break;
    const int copy = kSym ? i / a.n0 : 0;
    const bool ppo_row = a.aug || copy == 0;
    float mu[2], sd[2], isd[2], raw[2], act[2], mt[2];
    float lp = 0.f, ent = 0.f, kl = 0.f, sym = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int j = lane + 32 * k;
      mu[k] = act[k] = mt[k] = 0.f;
      raw[k] = c_raw[k];
      sd[k] = c_sd[k];
      isd[k] = c_isd[k];
      float lsd = c_lsd[k];
      if (j < a.A) {
        mu[k] = pf_mu[rr][k];
        if (a.hetero) {
          raw[k] = pf_raw[rr][k];
          std_terms(raw[k], a, sd[k], lsd, isd[k]);
        }
        if (copy > 0) {  // mirror loss against the original's signed-permuted mean
          mt[k] = pf_mt[rr][k];
          const float dm = mu[k] - mt[k];
          sym += dm * dm;
        }
        act[k] = pf_act[rr][k];
        const float z = (act[k] - mu[k]) * isd[k];
        lp += -0.5f * z * z - lsd - kLogSqrt2Pi;
        if (copy == 0) {
          const float omu = pf_omu[rr][k];
          const float osd = pf_osd[rr][k];
          ent += 0.5f + kLogSqrt2Pi + lsd;
          // KL(old || new) for diagonal Gaussians; only compared against the adaptive-LR thresholds, so the fast
          // logarithm suffices: log(vr) = 2 log(osd / sd)
          const float r = osd * isd[k];
          const float t1 = (omu - mu[k]) * isd[k];
          kl += 0.5f * (r * r + t1 * t1 - 1.0f) - __logf(r);
        }
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      lp += __shfl_xor_sync(0xffffffffu, lp, off);
      ent += __shfl_xor_sync(0xffffffffu, ent, off);
      kl += __shfl_xor_sync(0xffffffffu, kl, off);
      sym += __shfl_xor_sync(0xffffffffu, sym, off);
    }
    float d_lp = 0.f, dv = 0.f, surr = 0.f, vloss = 0.f;
    if (ppo_row) {
      // surrogate (identical on every lane)
      const float adv = pf_adv[rr];
      const float ratio = expf(lp - pf_lp[rr]);
      const float lo = 1.0f - a.clip, hi = 1.0f + a.clip;
      const float rc = fminf(fmaxf(ratio, lo), hi);
      const float s1 = -adv * ratio, s2 = -adv * rc;
      float g1, g2;
      max_grad_split(s1, s2, g1, g2);
      const float in_rng = (ratio >= lo && ratio <= hi) ? 1.f : 0.f;
      const float d_ratio = (g1 * -adv + g2 * -adv * in_rng) * invP;
      d_lp = d_ratio * ratio;
      surr = fmaxf(s1, s2);
      // value loss
      const float v = pf_v[rr];
      const float ret = pf_ret[rr];
      const float vold = pf_vold[rr];
      if (a.clipped_value) {
        const float dvv = v - vold;
        const float vc = vold + fminf(fmaxf(dvv, -a.clip), a.clip);
        const float l1 = (v - ret) * (v - ret), l2 = (vc - ret) * (vc - ret);
        float q1, q2;
        max_grad_split(l1, l2, q1, q2);
        const float vin = (dvv >= -a.clip && dvv <= a.clip) ? 1.f : 0.f;
        vloss = fmaxf(l1, l2);
        dv = q1 * 2.f * (v - ret) + q2 * 2.f * (vc - ret) * vin;
      } else {
        vloss = (ret - v) * (ret - v);
        dv = 2.f * (v - ret);
      }
      dv *= a.value_coef * invP;
    }
    const float ent_w = copy == 0 ? a.entropy_coef * invE : 0.f;
    const float mir_w = copy > 0 ? 2.f * a.mirror_coef * invM : 0.f;
    // gradients w.r.t. mean and std of each action
    __nv_bfloat16* dh = static_cast<__nv_bfloat16*>(a.d_head) + static_cast<size_t>(i) * a.ld_dhead;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int j = lane + 32 * k;
      if (j < a.A) {
        const float inv_var = isd[k] * isd[k];
        const float diff = act[k] - mu[k];
        const float dmu = d_lp * diff * inv_var + mir_w * (mu[k] - mt[k]);
        const float dsd = (d_lp * (diff * diff * inv_var - 1.0f) - ent_w) * isd[k];
        // chain through the std parameterisation (clamp passes the gradient on [lo, hi] inclusive)
        float dsd_raw;
        if (a.log_std) {
          const float in = (raw[k] >= a.log_std_lo && raw[k] <= a.log_std_hi) ? 1.f : 0.f;
          dsd_raw = dsd * sd[k] * in;
        } else {
          const float in = (raw[k] >= a.std_lo && raw[k] <= a.std_hi) ? 1.f : 0.f;
          dsd_raw = dsd * in;
        }
        dh[j] = __float2bfloat16_rn(dmu);
        acc_dh[k] += dmu;
        if (a.hetero) {
          dh[a.A + j] = __float2bfloat16_rn(dsd_raw);
          acc_dh[2 + k] += dsd_raw;
        } else {
          acc_dstd[k] += dsd_raw;
        }
      }
    }
    // zero the padding columns of the head gradient
    for (int c = head_cols + lane; c < a.ld_dhead; c += 32) dh[c] = __float2bfloat16_rn(0.f);
    if (lane == 0) {
      if (ppo_row) {
        __nv_bfloat16* dvp = static_cast<__nv_bfloat16*>(a.d_value) + static_cast<size_t>(i) * a.ld_dvalue;
        dvp[0] = __float2bfloat16_rn(dv);
        for (int c = 1; c < a.ld_dvalue; ++c) dvp[c] = __float2bfloat16_rn(0.f);
        acc_surr += surr * invP;
        acc_val += vloss * invP;
        acc_dv += dv;
      }
      if (copy == 0) {
        acc_ent += ent * invE;
        acc_kl += kl * invE;
      }
      acc_sym += sym * invM;
    }
  }
  }  // row groups
  // ---- block reduction in fixed warp order ----
  __shared__ float sh_dh[kLossWarps][4][32];
  __shared__ float sh_dstd[kLossWarps][2][32];
  __shared__ float sh_sc[kLossWarps][kLossStats + 1];
#pragma unroll
  for (int k = 0; k < 4; ++k) sh_dh[warp][k][lane] = acc_dh[k];
  sh_dstd[warp][0][lane] = acc_dstd[0];
  sh_dstd[warp][1][lane] = acc_dstd[1];
  if (lane == 0) {
    sh_sc[warp][0] = acc_surr;
    sh_sc[warp][1] = acc_val;
    sh_sc[warp][2] = acc_ent;
    sh_sc[warp][3] = acc_kl;
    sh_sc[warp][4] = acc_sym;
    sh_sc[warp][5] = acc_dv;
  }
  __syncthreads();
  const int t = threadIdx.x;
  if (t < 64) {
    // mean-gradient column sums (cols 0..A-1) and hetero std columns (A..2A-1)
    const int k = t >> 5, l = t & 31;
    const int j = 32 * k + l;
    float s = 0.f, sstd = 0.f, sraw = 0.f;
    for (int w = 0; w < kLossWarps; ++w) {
      s += sh_dh[w][k][l];
      sstd += sh_dstd[w][k][l];
      sraw += sh_dh[w][2 + k][l];
    }
    if (j < a.A) {
      a.dhead_colsum[static_cast<size_t>(blockIdx.x) * head_cols + j] = s;
      if (a.hetero)
        a.dhead_colsum[static_cast<size_t>(blockIdx.x) * head_cols + a.A + j] = sraw;
      else if (a.dstd_partial)
        a.dstd_partial[static_cast<size_t>(blockIdx.x) * a.A + j] = sstd;
    }
  } else if (t < 64 + kLossStats + 1) {
    const int q = t - 64;
    float s = 0.f;
    for (int w = 0; w < kLossWarps; ++w) s += sh_sc[w][q];
    if (q < kLossStats)
      a.stats_partial[static_cast<size_t>(blockIdx.x) * kLossStats + q] = s;
    else
      a.dvalue_colsum[blockIdx.x] = s;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// PPO loss without symmetry copies (the common path): eight lanes per row, four rows per warp
// ---------------------------------------------------------------------------------------------------------------
// Lane l8 = lane % 8 of row group g = lane / 8 holds actions 4 l8 .. 4 l8 + 3 (A <= 32). The row's scalar terms
// (ratio, clipped surrogate, clipped value loss) are evaluated once per eight lanes instead of once per 32, the
// per-row sums need three shuffle rounds, and every load of a row is issued before its arithmetic. Same formulas and
// tie rules as ppo_loss_kernel; the per-block partials have the same layout (grid = ppo_loss_blocks(B)).
constexpr int kLoss8Warps = 8;
static_assert(kLoss8Warps * 4 == kLossRowsPerBlock, "row groups of the two loss kernels must match");

__global__ void __launch_bounds__(kLoss8Warps * 32, 2) ppo_loss_rows8_kernel(const PpoLossArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 3;   // row of the warp's four
  const int l8 = lane & 7;   // action group
  const float invP = 1.0f / static_cast<float>(a.n0);
  const float invE = invP;
  const int A = a.A;
  const int head_cols = a.hetero ? 2 * A : A;
  float acc_dh[4] = {0.f, 0.f, 0.f, 0.f}, acc_ds[4] = {0.f, 0.f, 0.f, 0.f};
  float acc_surr = 0.f, acc_val = 0.f, acc_ent = 0.f, acc_kl = 0.f, acc_dv = 0.f;
  // state-independent std of this lane's actions (a parameter), once per kernel
  float c_raw[4], c_sd[4], c_lsd[4], c_isd[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int j = 4 * l8 + k;
    c_raw[k] = (!a.hetero && j < A) ? a.std_param[j] : 1.f;
    std_terms(c_raw[k], a, c_sd[k], c_lsd[k], c_isd[k]);
  }
  const int ngroups = (a.B + kLossRowsPerBlock - 1) / kLossRowsPerBlock;
  for (int grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
    const int i = grp * kLossRowsPerBlock + warp * 4 + g;
    const bool in = i < a.B;  // rows past B still take part in the warp's shuffles, with neutral values
    int src = in ? a.idx[i] : 0;
    RL_CHECK_INDEX(src, a.total, a.status, 44);
    const float* h = a.head + static_cast<size_t>(in ? i : 0) * a.ld_head;
    // ---- loads ----
    float act[4], omu[4], osd[4], mu[4], raw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * l8 + k;
      const bool ok = in && j < A;
      const size_t so = static_cast<size_t>(src) * A + j;
      act[k] = ok ? a.st_actions[so] : 0.f;
      omu[k] = ok ? a.st_mean[so] : 0.f;
      osd[k] = ok ? a.st_std[so] : 1.f;
      mu[k] = ok ? h[j] : 0.f;
      raw[k] = (ok && a.hetero) ? h[A + j] : c_raw[k];
    }
    const float adv = !in ? 0.f : (a.adv_override ? a.adv_override[i] : a.st_adv[src]);
    const float lp_old = in ? a.st_logp[src] : 0.f;
    const float ret = in ? a.st_ret[src] : 0.f;
    const float vold = in ? a.st_val[src] : 0.f;
    const float v = in ? a.value[static_cast<size_t>(i) * a.ld_value] : 0.f;
    // ---- per-action terms ----
    float sd[4], isd[4], lp = 0.f, ent = 0.f, kl = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * l8 + k;
      sd[k] = c_sd[k];
      isd[k] = c_isd[k];
      float lsd = c_lsd[k];
      if (a.hetero) std_terms(raw[k], a, sd[k], lsd, isd[k]);
      if (in && j < A) {
        const float z = (act[k] - mu[k]) * isd[k];
        lp += -0.5f * z * z - lsd - kLogSqrt2Pi;
        ent += 0.5f + kLogSqrt2Pi + lsd;
        const float r = osd[k] * isd[k];
        const float t1 = (omu[k] - mu[k]) * isd[k];
        kl += 0.5f * (r * r + t1 * t1 - 1.0f) - __logf(r);
      }
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      lp += __shfl_xor_sync(0xffffffffu, lp, off);
      ent += __shfl_xor_sync(0xffffffffu, ent, off);
      kl += __shfl_xor_sync(0xffffffffu, kl, off);
    }
    // ---- row terms (identical on the row's eight lanes) ----
    const float ratio = expf(lp - lp_old);
    const float lo = 1.0f - a.clip, hi = 1.0f + a.clip;
    const float rc = fminf(fmaxf(ratio, lo), hi);
    const float s1 = -adv * ratio, s2 = -adv * rc;
    float g1, g2;
    max_grad_split(s1, s2, g1, g2);
    const float in_rng = (ratio >= lo && ratio <= hi) ? 1.f : 0.f;
    const float d_lp = (g1 * -adv + g2 * -adv * in_rng) * invP * ratio;
    const float surr = fmaxf(s1, s2);
    float dv, vloss;
    if (a.clipped_value) {
      const float dvv = v - vold;
      const float vc = vold + fminf(fmaxf(dvv, -a.clip), a.clip);
      const float l1 = (v - ret) * (v - ret), l2 = (vc - ret) * (vc - ret);
      float q1, q2;
      max_grad_split(l1, l2, q1, q2);
      const float vin = (dvv >= -a.clip && dvv <= a.clip) ? 1.f : 0.f;
      vloss = fmaxf(l1, l2);
      dv = q1 * 2.f * (v - ret) + q2 * 2.f * (vc - ret) * vin;
    } else {
      vloss = (ret - v) * (ret - v);
      dv = 2.f * (v - ret);
    }
    dv *= a.value_coef * invP;
    const float ent_w = a.entropy_coef * invE;
    // ---- gradients w.r.t. mean and std ----
    float dmu[4], dsr[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * l8 + k;
      dmu[k] = dsr[k] = 0.f;
      if (in && j < A) {
        const float inv_var = isd[k] * isd[k];
        const float diff = act[k] - mu[k];
        dmu[k] = d_lp * diff * inv_var;
        const float dsd = (d_lp * (diff * diff * inv_var - 1.0f) - ent_w) * isd[k];
        if (a.log_std) {
          const float in = (raw[k] >= a.log_std_lo && raw[k] <= a.log_std_hi) ? 1.f : 0.f;
          dsr[k] = dsd * sd[k] * in;
        } else {
          const float in = (raw[k] >= a.std_lo && raw[k] <= a.std_hi) ? 1.f : 0.f;
          dsr[k] = dsd * in;
        }
        acc_dh[k] += dmu[k];
        acc_ds[k] += dsr[k];
      }
    }
    if (!in) continue;  // past this point only the row's own stores and accumulators
    __nv_bfloat16* dh = static_cast<__nv_bfloat16*>(a.d_head) + static_cast<size_t>(i) * a.ld_dhead;
    if (!a.hetero) {
      // columns 4 l8 .. 4 l8 + 3 in one 8-byte store (zeros past A: the padding columns of the row)
      if (4 * l8 < a.ld_dhead)
        *reinterpret_cast<uint2*>(dh + 4 * l8) = make_uint2(pack_bf16x2(dmu[0], dmu[1]), pack_bf16x2(dmu[2], dmu[3]));
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = 4 * l8 + k;
        if (j < A) {
          dh[j] = __float2bfloat16_rn(dmu[k]);
          dh[A + j] = __float2bfloat16_rn(dsr[k]);
        }
      }
    }
    for (int c = (a.hetero ? head_cols : 32) + l8; c < a.ld_dhead; c += 8) dh[c] = __float2bfloat16_rn(0.f);
    if (l8 == 0) {
      __nv_bfloat16* dvp = static_cast<__nv_bfloat16*>(a.d_value) + static_cast<size_t>(i) * a.ld_dvalue;
      if (a.ld_dvalue == 8) {
        *reinterpret_cast<uint4*>(dvp) = make_uint4(pack_bf16x2(dv, 0.f), 0u, 0u, 0u);
      } else {
        dvp[0] = __float2bfloat16_rn(dv);
        for (int c = 1; c < a.ld_dvalue; ++c) dvp[c] = __float2bfloat16_rn(0.f);
      }
      acc_surr += surr * invP;
      acc_val += vloss * invP;
      acc_dv += dv;
      acc_ent += ent * invE;
      acc_kl += kl * invE;
    }
  }
  // ---- block reduction in a fixed order: row groups of a warp, then warps ----
#pragma unroll
  for (int off = 8; off < 32; off <<= 1) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      acc_dh[k] += __shfl_xor_sync(0xffffffffu, acc_dh[k], off);
      acc_ds[k] += __shfl_xor_sync(0xffffffffu, acc_ds[k], off);
    }
    acc_surr += __shfl_xor_sync(0xffffffffu, acc_surr, off);
    acc_val += __shfl_xor_sync(0xffffffffu, acc_val, off);
    acc_ent += __shfl_xor_sync(0xffffffffu, acc_ent, off);
    acc_kl += __shfl_xor_sync(0xffffffffu, acc_kl, off);
    acc_dv += __shfl_xor_sync(0xffffffffu, acc_dv, off);
  }
  __shared__ float sh_dh[kLoss8Warps][32];
  __shared__ float sh_ds[kLoss8Warps][32];
  __shared__ float sh_sc[kLoss8Warps][kLossStats + 1];
  if (lane < 8) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      sh_dh[warp][4 * lane + k] = acc_dh[k];
      sh_ds[warp][4 * lane + k] = acc_ds[k];
    }
  }
  if (lane == 0) {
    sh_sc[warp][0] = acc_surr;
    sh_sc[warp][1] = acc_val;
    sh_sc[warp][2] = acc_ent;
    sh_sc[warp][3] = acc_kl;
    sh_sc[warp][4] = 0.f;  // no mirror loss without copies
    sh_sc[warp][5] = acc_dv;
  }
  __syncthreads();
  const int t = threadIdx.x;
  if (t < 32) {
    float sdh = 0.f, sds = 0.f;
#pragma unroll
    for (int w = 0; w < kLoss8Warps; ++w) {
      sdh += sh_dh[w][t];
      sds += sh_ds[w][t];
    }
    if (t < A) {
      a.dhead_colsum[static_cast<size_t>(blockIdx.x) * head_cols + t] = sdh;
      if (a.hetero)
        a.dhead_colsum[static_cast<size_t>(blockIdx.x) * head_cols + A + t] = sds;
      else if (a.dstd_partial)
        a.dstd_partial[static_cast<size_t>(blockIdx.x) * A + t] = sds;
    }
  } else if (t < 32 + kLossStats + 1) {
    const int q = t - 32;
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kLoss8Warps; ++w) sum += sh_sc[w][q];
    if (q < kLossStats)
      a.stats_partial[static_cast<size_t>(blockIdx.x) * kLossStats + q] = sum;
    else
      a.dvalue_colsum[blockIdx.x] = sum;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Behaviour-cloning loss gradient: one warp per row (lane j: columns j, j + 32), 8 warps x 4 rows per block
// ---------------------------------------------------------------------------------------------------------------
constexpr int kMseWarps = 8;
constexpr int kMseRowsPerWarp = 4;
constexpr int kMseRowsPerBlock = kMseWarps * kMseRowsPerWarp;

__global__ void __launch_bounds__(kMseWarps * 32) mse_grad_kernel(const MseArgs a) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float w_last = a.last_weight ? *a.last_weight : 1.0f;
  const float n_rows = a.denom_rows > 0 ? static_cast<float>(a.denom_rows) : static_cast<float>(a.rows - 1) + w_last;
  const float inv_n = 1.0f / (n_rows * static_cast<float>(a.A));
  float col[2] = {0.f, 0.f};
  float loss = 0.f;
  const int ngroups = (a.rows + kMseRowsPerBlock - 1) / kMseRowsPerBlock;
  for (int grp = blockIdx.x; grp < ngroups; grp += gridDim.x)
  for (int r = 0; r < kMseRowsPerWarp; ++r) {
    const int i = grp * kMseRowsPerBlock + warp * kMseRowsPerWarp + r;
    if (i >= a.rows) break;
    __nv_bfloat16* g = static_cast<__nv_bfloat16*>(a.grad) + static_cast<size_t>(i) * a.ld_grad;
    const float w = i == a.rows - 1 ? w_last : 1.0f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int j = lane + 32 * k;
      if (j < a.A) {
        const float d = a.pred[static_cast<size_t>(i) * a.ld_pred + j] - a.target[static_cast<size_t>(i) * a.ld_target + j];
        float gd;
        if (a.huber) {  // torch huber_loss, delta = 1: 0.5 d^2 inside |d| < 1, |d| - 0.5 outside
          const float ad = fabsf(d);
          loss += w * (ad < 1.f ? 0.5f * d * d : ad - 0.5f);
          gd = fminf(fmaxf(d, -1.f), 1.f) * (w * inv_n);
        } else {
          loss += w * (d * d);
          gd = 2.f * d * (w * inv_n);
        }
        g[j] = __float2bfloat16_rn(gd);
        col[k] += gd;
      } else if (j < a.ld_grad) {
        g[j] = __float2bfloat16_rn(0.f);
      }
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) loss += __shfl_xor_sync(0xffffffffu, loss, off);
  __shared__ float s_col[kMseWarps][64];
  __shared__ float s_loss[kMseWarps];
  __shared__ bool s_last;
  s_col[warp][lane] = col[0];
  s_col[warp][lane + 32] = col[1];
  if (lane == 0) s_loss[warp] = loss;
  __syncthreads();
  if (threadIdx.x < a.head_cols) {
    float c = 0.f;
    for (int w = 0; w < kMseWarps; ++w) c += s_col[w][threadIdx.x];
    a.colsum_partial[static_cast<size_t>(blockIdx.x) * a.head_cols + threadIdx.x] = c;
  }
  if (threadIdx.x == 0) {
    float l = 0.f;
    for (int w = 0; w < kMseWarps; ++w) l += s_loss[w];
    a.loss_partial[blockIdx.x] = l;
    __threadfence();
    s_last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || warp != 0) return;
  // last block: fixed-order sum of the block partials (lane-strided, then a butterfly)
  __threadfence();
  float t = 0.f;
  for (int b = lane; b < static_cast<int>(gridDim.x); b += 32) t += __ldcg(a.loss_partial + b);
#pragma unroll
  for (int off = 16; off; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
  if (lane == 0) {
    *a.loss_acc += t * inv_n;
    *a.ticket = 0u;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// segment reduction (sum of partial slabs in fixed order, fp64 accumulation)
// ---------------------------------------------------------------------------------------------------------------
// One warp per chunk of 32 columns (lane = column, coalesced 128-byte rows), warps striding over the chunks of all
// segments. A lane keeps 8 loads of its column in flight (parts p .. p + 7) and adds them into four fp64 partial
// sums in a fixed order, so the result is deterministic for any launch configuration; a GPU-wide grid of such warps
// keeps enough bytes in flight to stream the partial slabs at HBM bandwidth.
constexpr int kReduceWarps = 8;
__global__ void __launch_bounds__(kReduceWarps * 32)
    reduce_segments_kernel(const ReduceSegment* __restrict__ segs, int nseg, int total_chunks, float* send0,
                           float* send1, const unsigned int* epoch, int accumulate) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  float* dst_base = (((epoch ? *epoch : 0u) + 1u) & 1u) ? send1 : send0;
  const int warps = gridDim.x * kReduceWarps;
  int s = 0;
  for (int chunk = blockIdx.x * kReduceWarps + (threadIdx.x >> 5); chunk < total_chunks; chunk += warps) {
    while (s + 1 < nseg && segs[s + 1].first_chunk <= chunk) ++s;  // chunks only grow along a warp's walk
    const ReduceSegment g = segs[s];
    const long long e = static_cast<long long>(chunk - g.first_chunk) * kReduceChunk + lane;
    if (e >= g.n) continue;
    const float* col = g.src + e;
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
    int p = 0;
    for (; p + 8 <= g.parts; p += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcs(col + static_cast<size_t>(p + u) * g.n);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u & 3] += v[u];
    }
    for (; p < g.parts; ++p) acc[0] += __ldcs(col + static_cast<size_t>(p) * g.n);
    const float t = static_cast<float>((acc[0] + acc[1]) + (acc[2] + acc[3]));
    float* dst = dst_base + g.dst_offset + e;
    *dst = accumulate ? *dst + t : t;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Grid barrier for co-resident (cooperatively launched) grids; bounded wait.
// ---------------------------------------------------------------------------------------------------------------
__device__ bool grid_sync(unsigned int* bar, unsigned int* status, uint64_t timeout_ns) {
  __syncthreads();
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    volatile unsigned int* gen = bar + 1;
    const unsigned int g = *gen;
    __threadfence();
    const unsigned int arrived = atomicAdd(bar, 1u) + 1u;
    if (arrived == gridDim.x) {
      atomicExch(bar, 0u);
      __threadfence();
      atomicAdd(bar + 1, 1u);
    } else {
      const uint64_t t0 = globaltimer_ns();
      while (*gen == g) {
        __nanosleep(64);
        if (globaltimer_ns() - t0 > timeout_ns) {
          report_error(status, kTimeoutGridBarrier, 50);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  return ok != 0;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Threads r < world wait, in parallel, until slot r of this rank's flag array reaches `target` (a bounded wait);
// returns false in every thread of the block if one slot did not arrive in time (site + r recorded).
__device__ bool await_peer_flags(const unsigned int* my_flags, int world, unsigned int target, uint64_t timeout_ns,
                                 unsigned int* status, int site, unsigned int* abort_word, unsigned int abort_tag) {
  __shared__ int all_arrived;
  if (threadIdx.x == 0) all_arrived = 1;
  __syncthreads();
  if (threadIdx.x < world) {
    const uint64_t t0 = globaltimer_ns();
    while (static_cast<int>(ld_acquire_sys(my_flags + threadIdx.x) - target) < 0) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        report_error(status, kTimeoutPeerFlag, site + threadIdx.x);
        all_arrived = 0;
        atomicExch(abort_word, abort_tag);  // grid-wide abort of this exchange (tagged with the epoch)
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  return all_arrived != 0;
}

// Thread r < world of the calling block stores `value` into slot `rank` of rank r's flag array (release).
__device__ __forceinline__ void publish_flag(unsigned int* const* peer_flags, int world, int rank, unsigned int value) {
  if (threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(peer_flags[threadIdx.x] + rank, value);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Fused exchange + clip + adaptive LR + Adam
// One-shot (world 2, or forced): every block publishes/awaits the epoch flags, then sums every element's gradient over
//          all ranks in rank order (bit-identical on every rank), divides by the world size, accumulates per-group
//          squared norms; after a grid barrier every block reduces the norm partials in the same order.
// Two-shot (world >= 2 with peer_reduced): flag round 1 (gradients sent), each rank averages only its own shard of
//          the vector over all ranks into its reduced buffer with the shard's squared norms; the last block to finish
//          sums the blocks' norm partials into the rank's norm slots and publishes flag round 2 (shard averaged);
//          after round 2 every rank sums the ranks' norm slots in rank order and reads each element's average from
//          its owner while it applies Adam. Peer bytes per rank: 2 (W - 1) / W of the vector instead of (W - 1).
// Both: the clip coefficients, the adapted learning rate and Adam follow; bf16 weight shadows are refreshed.
// Every flag wait is bounded; the ranks' flags are polled in parallel (one thread per rank).
// ---------------------------------------------------------------------------------------------------------------
constexpr int kAdamThreads = 256;
constexpr int kMaxWorldAdam = 8;

// Two-shot exchange: copy elements [e0, e0 + n) of the rank-averaged gradient from their owners' reduced buffers into
// a.grads with 16-byte peer loads (a float4 never straddles two shards); the calling block then reads them locally.
__device__ void gather_owned(const AdamArgs& a, long long e0, long long n) {
  const long long e1 = e0 + n;
  const long long a0 = (e0 + 3) & ~3ll, a1 = e1 & ~3ll;  // aligned body [a0, a1)
  for (long long e = e0 + threadIdx.x; e < (a0 < e1 ? a0 : e1); e += blockDim.x)
    a.grads[e] = __ldcv(a.peer_reduced[(e >> 2) / a.shard4] + e);
  for (long long v = (a0 >> 2) + threadIdx.x; v < (a1 >> 2); v += blockDim.x)
    reinterpret_cast<float4*>(a.grads)[v] = __ldcv(reinterpret_cast<const float4*>(a.peer_reduced[v / a.shard4]) + v);
  for (long long e = (a1 > a0 ? a1 : a0) + threadIdx.x; e < e1; e += blockDim.x)
    a.grads[e] = __ldcv(a.peer_reduced[(e >> 2) / a.shard4] + e);
}

// Clip coefficients, adapted learning rate and Adam constants from the global squared norms `norm_sq` (identical in
// every block and on every rank), then Adam over this block's chunks reading the rank-averaged gradient from a.grads.
// With `gather` (the two-shot exchange) each chunk's gradient is first copied there from its owners by the same
// block. Block 0 finally advances the step counters, learning rates and the epoch.
__device__ void adam_apply(const AdamArgs& a, const float* norm_sq, float kl, unsigned int epoch,
                           const long long* step_s, const float* lr_old, bool exchange_ok, bool gather) {
  __shared__ float coef[kAdamMaxGroups], lr_s[kAdamMaxGroups];
  __shared__ float step_size_s[kAdamMaxGroups], bc2_sqrt_s[kAdamMaxGroups];
  if (threadIdx.x < a.ngroups) {
    const int g = threadIdx.x;
    const float norm = sqrtf(norm_sq[g]);
    coef[g] = a.max_norm[g] > 0.f ? fminf(a.max_norm[g] / (norm + 1e-6f), 1.0f) : 1.0f;
    float lr = lr_old[g];  // slot g
    if (g == 0 && a.adaptive) {
      if (kl > a.desired_kl * 2.0f)
        lr = fmaxf(a.lr_min, lr / 1.5f);
      else if (kl < a.desired_kl / 2.0f && kl > 0.0f)
        lr = fminf(a.lr_max, lr * 1.5f);
    }
    lr_s[g] = lr;
    if (blockIdx.x == 0 && a.out_norms) a.out_norms[g] = norm;
  }
  __syncthreads();
  if (!exchange_ok) {  // leave parameters untouched when the exchange failed; the status word reports it
    if (blockIdx.x == 0 && threadIdx.x == 0) *a.epoch = epoch;
    return;
  }
  // per-group Adam constants (bias corrections in double, as torch computes them on the host)
  if (threadIdx.x < a.ngroups) {
    const int g = threadIdx.x;
    const double step = static_cast<double>(step_s[g] + 1);
    const double bc1 = 1.0 - pow(static_cast<double>(a.beta1[g]), step);
    const double bc2 = 1.0 - pow(static_cast<double>(a.beta2[g]), step);
    step_size_s[g] = static_cast<float>(static_cast<double>(lr_s[a.lr_index[g]]) / bc1);
    bc2_sqrt_s[g] = static_cast<float>(sqrt(bc2));
  }
  __syncthreads();
  for (int c = blockIdx.x; c < a.nchunks; c += gridDim.x) {
    const AdamChunk ch = a.chunks[c];
    const AdamTensor T = a.tensors[ch.tensor];
    const int g = T.group;
    if (gather) {  // block-uniform: every thread of the block takes part before any reads the chunk
      gather_owned(a, T.offset + ch.start, ch.count);
      __syncthreads();
    }
    if (g < 0) continue;  // exchanged statistics (e.g. the KL mean), not parameters
    const float step_size = step_size_s[g], bc2_sqrt = bc2_sqrt_s[g];
    const float b1 = a.beta1[g], b2 = a.beta2[g], eps = a.eps[g], cf = coef[g];
    for (int k = threadIdx.x; k < ch.count; k += blockDim.x) {
      const long long e = T.offset + ch.start + k;
      const float grad = a.grads[e] * cf;
      float m = a.exp_avg[e];
      m = m + (1.0f - b1) * (grad - m);
      const float v = b2 * a.exp_avg_sq[e] + (1.0f - b2) * grad * grad;
      const float denom = sqrtf(v) / bc2_sqrt + eps;
      const float p = a.params[e] - step_size * (m / denom);
      a.exp_avg[e] = m;
      a.exp_avg_sq[e] = v;
      a.params[e] = p;
      if (T.shadow) {
        const unsigned int idx = static_cast<unsigned int>(ch.start + k);
        const unsigned int r = T.cols_shift == 32 ? idx : __umulhi(idx, T.cols_magic) >> T.cols_shift;  // idx / cols
        const unsigned int col = idx - r * static_cast<unsigned int>(T.cols);
        static_cast<__nv_bfloat16*>(T.shadow)[static_cast<size_t>(r) * T.shadow_ld + col] = __float2bfloat16_rn(p);
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < a.ngroups) {
    a.lr[threadIdx.x] = lr_s[threadIdx.x];
    a.step[threadIdx.x] = step_s[threadIdx.x] + 1;
    if (threadIdx.x == 0) {
      *a.epoch = epoch;
      if (a.lr_out_slot) *a.lr_out_slot = lr_s[0];
    }
  }
}

// Per-group squared norms of the float4 `g` of elements 4 v .. 4 v + 3, added into sq.
__device__ __forceinline__ void add_group_squares(const AdamArgs& a, long long v, float4 g, float* sq) {
  const long long e = 4 * v;
  const float comp[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
#pragma unroll
    for (int gr = 0; gr < kAdamMaxGroups; ++gr)
      if (gr < a.ngroups && e + c >= a.group_begin[gr] && e + c < a.group_end[gr]) sq[gr] += comp[c] * comp[c];
  }
}

// Block sum (fixed warp order) of the per-thread group squares into red[0..kAdamMaxGroups) of thread 0's view.
__device__ __forceinline__ void block_group_sums(float* sq, float (*red)[kAdamMaxGroups]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int g = 0; g < kAdamMaxGroups; ++g) {
#pragma unroll
    for (int off = 16; off; off >>= 1) sq[g] += __shfl_xor_sync(0xffffffffu, sq[g], off);
  }
  __syncthreads();  // red[] may still be read by a previous use
  if (lane == 0)
    for (int g = 0; g < kAdamMaxGroups; ++g) red[warp][g] = sq[g];
  __syncthreads();
}

__device__ __forceinline__ float4 rank_average(const AdamArgs& a, unsigned int parity, long long v, float inv_world) {
  float4 part[kMaxWorldAdam];
#pragma unroll
  for (int r = 0; r < kMaxWorldAdam; ++r)  // every rank's loads in flight before the rank-ordered sum
    if (r < a.world) part[r] = __ldcv(reinterpret_cast<const float4*>(a.peer_send[parity * a.world + r]) + v);
  float4 g = part[0];
#pragma unroll
  for (int r = 1; r < kMaxWorldAdam; ++r) {
    if (r < a.world) {
      g.x += part[r].x;
      g.y += part[r].y;
      g.z += part[r].z;
      g.w += part[r].w;
    }
  }
  g.x *= inv_world;
  g.y *= inv_world;
  g.z *= inv_world;
  g.w *= inv_world;
  return g;
}

__device__ void adam_two_shot(const AdamArgs& a, unsigned int epoch, const long long* step_s, const float* lr_old) {
  __shared__ float red[kAdamThreads / 32][kAdamMaxGroups];
  __shared__ float norm_sq[kAdamMaxGroups];
  __shared__ unsigned int ticket_s;
  const unsigned int round1 = 2u * epoch, round2 = 2u * epoch + 1u;
  // ---- round 1: this rank's gradients are in its send buffer ----
  if (blockIdx.x == 0) publish_flag(a.peer_flags, a.world, a.rank, round1);
  bool ok = await_peer_flags(a.peer_flags[a.rank], a.world, round1, a.timeout_ns, a.status, 60, a.barrier + 2, epoch);
  // ---- reduce-scatter: the own shard, averaged over the ranks in rank order ----
  float sq[kAdamMaxGroups] = {0.f, 0.f, 0.f, 0.f};
  const unsigned int parity = epoch & 1u;
  const float inv_world = 1.0f / static_cast<float>(a.world);
  const long long n4 = a.exchange_len / 4;
  const long long v0 = static_cast<long long>(a.rank) * a.shard4;
  const long long v1 = v0 + a.shard4 < n4 ? v0 + a.shard4 : n4;
  float4* mine = reinterpret_cast<float4*>(a.peer_reduced[a.rank]);
  if (ok) {
    for (long long v = v0 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; v < v1;
         v += static_cast<long long>(gridDim.x) * blockDim.x) {
      const float4 g = rank_average(a, parity, v, inv_world);
      mine[v] = g;
      add_group_squares(a, v, g, sq);
    }
  }
  block_group_sums(sq, red);
  if (threadIdx.x < kAdamMaxGroups) {
    float t = 0.f;
    for (int w = 0; w < kAdamThreads / 32; ++w) t += red[w][threadIdx.x];
    a.norm_partial[static_cast<size_t>(blockIdx.x) * kAdamMaxGroups + threadIdx.x] = t;
  }
  // the last block to finish sums the blocks' partials (block order) into this rank's norm slots and opens round 2
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) ticket_s = atomicAdd(a.barrier + 3, 1u);
  __syncthreads();
  if (ticket_s == gridDim.x - 1) {
    __threadfence();
    if (threadIdx.x < kAdamMaxGroups) {
      float t = 0.f;
      for (int b = 0; b < static_cast<int>(gridDim.x); ++b)
        t += __ldcg(a.norm_partial + static_cast<size_t>(b) * kAdamMaxGroups + threadIdx.x);
      reinterpret_cast<float*>(mine)[a.exchange_len + threadIdx.x] = t;
    }
    if (threadIdx.x == 0) atomicExch(a.barrier + 3, 0u);
    __syncthreads();
    // a block whose round-1 wait gave up tagged the abort word before its ticket: then the shard was not averaged,
    // round 2 is not opened, and the peers' round-2 waits give up as well
    if (*reinterpret_cast<volatile unsigned int*>(a.barrier + 2) != epoch)
      publish_flag(a.peer_flags, a.world, a.rank, round2);
  }
  // ---- round 2: every shard is averaged; global norms from the ranks' slots in rank order ----
  if (ok)
    ok = await_peer_flags(a.peer_flags[a.rank], a.world, round2, a.timeout_ns, a.status, 70, a.barrier + 2, epoch);
  ok = ok && *reinterpret_cast<volatile unsigned int*>(a.barrier + 2) != epoch;
  if (threadIdx.x < a.ngroups) {
    float t = 0.f;
    for (int r = 0; r < a.world; ++r) t += __ldcv(a.peer_reduced[r] + a.exchange_len + threadIdx.x);
    norm_sq[threadIdx.x] = t;
  }
  // the owner of element e holds its average: shard of float4 index e / 4
  __shared__ float kl_s;
  if (threadIdx.x == 0)
    kl_s = (a.adaptive && a.kl_offset >= 0 && ok) ? __ldcv(a.peer_reduced[(a.kl_offset >> 2) / a.shard4] + a.kl_offset)
                                                  : 0.f;
  __syncthreads();
  adam_apply(a, norm_sq, kl_s, epoch, step_s, lr_old, ok, true);
}

__global__ void __launch_bounds__(kAdamThreads) adam_step_kernel(const AdamArgs a) {
  __shared__ float red[kAdamThreads / 32][kAdamMaxGroups];
  __shared__ float norm_sq[kAdamMaxGroups];
  __shared__ long long step_s[kAdamMaxGroups];
  __shared__ float lr_old[kAdamMaxGroups];
  __shared__ unsigned int epoch_s;
  __shared__ int peers_ok;
  // Everything block 0 rewrites at the end (step, learning rates, epoch) is read here, before any block can finish.
  if (threadIdx.x == 0) {
    peers_ok = 1;
    for (int g = 0; g < a.ngroups; ++g) {
      step_s[g] = a.step[g];
      lr_old[g] = a.lr[g];
    }
    epoch_s = *a.epoch + 1u;
  }
  __syncthreads();
  const unsigned int epoch = epoch_s;
  if (a.world > 1 && a.peer_reduced != nullptr) {
    adam_two_shot(a, epoch, step_s, lr_old);
    return;
  }
  // ---- one-shot: flags ----
  if (a.world > 1) {
    // publish: this rank's slot in every peer's flag array (release orders our gradient writes before the flag)
    if (blockIdx.x == 0) publish_flag(a.peer_flags, a.world, a.rank, epoch);
    if (!await_peer_flags(a.peer_flags[a.rank], a.world, epoch, a.timeout_ns, a.status, 60, a.barrier + 2, epoch))
      peers_ok = 0;
  }
  __syncthreads();
  const bool exchange_ok = peers_ok != 0;
  // ---- rank-ordered sum of every element, squared norms ----
  float sq[kAdamMaxGroups] = {0.f, 0.f, 0.f, 0.f};
  const float inv_world = 1.0f / static_cast<float>(a.world);
  const unsigned int parity = epoch & 1u;
  const float4* mine4 = reinterpret_cast<const float4*>(a.send[parity]);
  const long long n4 = a.exchange_len / 4;
  for (long long v = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; v < n4;
       v += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 g = (a.world > 1 && exchange_ok) ? rank_average(a, parity, v, inv_world) : mine4[v];
    reinterpret_cast<float4*>(a.grads)[v] = g;
    add_group_squares(a, v, g, sq);
  }
  block_group_sums(sq, red);
  if (threadIdx.x < kAdamMaxGroups) {
    float t = 0.f;
    for (int w = 0; w < kAdamThreads / 32; ++w) t += red[w][threadIdx.x];
    a.norm_partial[static_cast<size_t>(blockIdx.x) * kAdamMaxGroups + threadIdx.x] = t;
  }
  if (!grid_sync(a.barrier, a.status, a.timeout_ns)) return;
  // every block takes the same decision: the exchange failed if any block's wait gave up
  const bool all_ok = *reinterpret_cast<volatile unsigned int*>(a.barrier + 2) != epoch;
  // every block reduces the per-block partials with all of its threads (fixed tree order: identical in every block)
  {
    float part[kAdamMaxGroups] = {0.f, 0.f, 0.f, 0.f};
    for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += blockDim.x) {
#pragma unroll
      for (int g = 0; g < kAdamMaxGroups; ++g) part[g] += a.norm_partial[static_cast<size_t>(b) * kAdamMaxGroups + g];
    }
    block_group_sums(part, red);
  }
  if (threadIdx.x < a.ngroups) {
    float t = 0.f;
    for (int w = 0; w < kAdamThreads / 32; ++w) t += red[w][threadIdx.x];
    norm_sq[threadIdx.x] = t;
  }
  const float kl = a.adaptive ? *a.kl_mean : 0.f;
  adam_apply(a, norm_sq, kl, epoch, step_s, lr_old, all_ok, false);
}


// ---------------------------------------------------------------------------------------------------------------
// Column statistics + EmpiricalNormalization update
// ---------------------------------------------------------------------------------------------------------------
constexpr int kStatsRowsPerChunk = 4096;
__global__ void colstats_kernel(const ColStatsArgs a) {
  // block (32 columns x 8 row lanes) per (column stripe, row chunk)
  const int col = blockIdx.x * 32 + threadIdx.x;
  const long long r0 = static_cast<long long>(blockIdx.y) * kStatsRowsPerChunk;
  const long long r1 = min(a.rows, r0 + kStatsRowsPerChunk);
  // four independent accumulator pairs, so four rows' loads are in flight per thread (the sums are combined in a
  // fixed order: deterministic)
  double s4[4] = {0.0, 0.0, 0.0, 0.0}, ss4[4] = {0.0, 0.0, 0.0, 0.0};
  if (col < a.dim) {
    const long long step = blockDim.y;
    long long r = r0 + threadIdx.y;
    for (; r + 3 * step < r1; r += 4 * step) {
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = __ldg(a.x + static_cast<size_t>(r + k * step) * a.ld + col);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const double d = v[k];
        s4[k] += d;
        ss4[k] += d * d;
      }
    }
    for (; r < r1; r += step) {
      const double d = __ldg(a.x + static_cast<size_t>(r) * a.ld + col);
      s4[0] += d;
      ss4[0] += d * d;
    }
  }
  const double s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  const double ss = (ss4[0] + ss4[1]) + (ss4[2] + ss4[3]);
  __shared__ double sh[2][8][33];
  sh[0][threadIdx.y][threadIdx.x] = s;
  sh[1][threadIdx.y][threadIdx.x] = ss;
  __syncthreads();
  if (threadIdx.y == 0 && col < a.dim) {
    double ts = 0, tss = 0;
    for (int y = 0; y < static_cast<int>(blockDim.y); ++y) {
      ts += sh[0][y][threadIdx.x];
      tss += sh[1][y][threadIdx.x];
    }
    a.partial[(static_cast<size_t>(blockIdx.y) * 2) * a.dim + col] = ts;
    a.partial[(static_cast<size_t>(blockIdx.y) * 2 + 1) * a.dim + col] = tss;
  }
}

// One block of 32 x 32 threads: for each 32-column stripe, lane y sums chunks y, y + 32, ... of its column, the 32
// partial sums are combined in a fixed order, then the running statistics of that stripe are updated.
__global__ void __launch_bounds__(1024) norm_update_kernel(const NormUpdateArgs a) {
  __shared__ long long count0;
  __shared__ int skip;
  __shared__ double red[2][32][33];
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    count0 = *a.count;
    skip = (a.until >= 0 && count0 >= a.until && !a.reduce_only) ? 1 : 0;
  }
  __syncthreads();
  if (skip) return;
  const double n = static_cast<double>(a.rows);
  const double new_count = static_cast<double>(count0) + n;
  const float rate = static_cast<float>(n / new_count);
  for (int c0 = 0; c0 < a.dim; c0 += 32) {
    const int c = c0 + threadIdx.x;
    double s = 0, ss = 0;
    if (c < a.dim) {
      for (int k = threadIdx.y; k < a.chunks; k += 32) {
        s += a.partial[(static_cast<size_t>(k) * 2) * a.dim + c];
        ss += a.partial[(static_cast<size_t>(k) * 2 + 1) * a.dim + c];
      }
    }
    red[0][threadIdx.y][threadIdx.x] = s;
    red[1][threadIdx.y][threadIdx.x] = ss;
    __syncthreads();
    if (threadIdx.y == 0 && c < a.dim) {
      double ts = 0, tss = 0;
      for (int y = 0; y < 32; ++y) {
        ts += red[0][y][threadIdx.x];
        tss += red[1][y][threadIdx.x];
      }
      if (a.moments_out) {
        a.moments_out[2 + c] = ts;
        a.moments_out[2 + a.dim + c] = tss;
      }
      if (!a.reduce_only) {
        const double bm = ts / n;
        const double bv = fmax(tss / n - bm * bm, 0.0);
        const float batch_mean = static_cast<float>(bm), batch_var = static_cast<float>(bv);
        const float old_mean = a.mean[c];
        const float delta = batch_mean - old_mean;
        const float new_mean = old_mean + rate * delta;
        const float new_var = a.var[c] + rate * (batch_var - a.var[c] + delta * (batch_mean - new_mean));
        a.mean[c] = new_mean;
        a.var[c] = new_var;
        a.std[c] = sqrtf(new_var);
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    if (a.moments_out) a.moments_out[0] = n;
    if (!a.reduce_only) *a.count = count0 + a.rows;
  }
}

__global__ void to_bf16_padded_kernel(const float* src, int rows, int cols, __nv_bfloat16* dst, int ld) {
  const long long total = static_cast<long long>(rows) * ld;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(e / ld), c = static_cast<int>(e - static_cast<long long>(r) * ld);
    dst[e] = __float2bfloat16_rn(c < cols ? src[static_cast<size_t>(r) * cols + c] : 0.f);
  }
}

int grid_for(long long work, int threads, int cap = 148 * 16) {
  long long g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return static_cast<int>(g);
}

}  // namespace

// ---------------------------------------------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------------------------------------------
cudaError_t prep_obs(const PrepObsArgs& a, cudaStream_t s) {
  int D = 0;
  for (int g = 0; g < a.groups; ++g) D += a.width[g];
  if (a.groups < 1 || a.groups > kMaxObsGroups || a.rows <= 0 || D > kPrepMaxD) return cudaErrorInvalidValue;
  launch_pdl(prep_obs_kernel, dim3(grid_for(a.rows, 8, 148 * 16)), dim3(256), 0, s, a, D);
  return cudaGetLastError();
}

cudaError_t gaussian_sample(const SampleArgs& a, cudaStream_t s) {
  if (a.A > 64 || a.rows <= 0) return cudaErrorInvalidValue;
  if (a.A <= 32)
    launch_pdl(gaussian_sample_rows8_kernel, dim3(grid_for(a.rows, 32)), dim3(256), 0, s, a);
  else
    launch_pdl(gaussian_sample_kernel, dim3(grid_for(a.rows, 8)), dim3(256), 0, s, a);
  return cudaGetLastError();
}

cudaError_t process_step(const ProcessArgs& a, cudaStream_t s) {
  launch_pdl(process_step_kernel, dim3(grid_for(a.rows, 256)), dim3(256), 0, s, a);
  return cudaGetLastError();
}

int gae_blocks(int N) { return (N + kGaeThreads - 1) / kGaeThreads; }

cudaError_t gae(const GaeArgs& a, cudaStream_t s) {
  gae_kernel<<<gae_blocks(a.N), kGaeThreads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t adv_normalize(float* adv, long long n, const double* partial, int parts, cudaStream_t s) {
  adv_normalize_kernel<<<grid_for(n, 256, 148 * 4), 256, 0, s>>>(adv, n, partial, parts);
  return cudaGetLastError();
}

uint32_t feistel_half_bits(long long total) {
  uint32_t bits = 2;
  while ((1ll << bits) < total) ++bits;
  return (bits + 1) / 2;
}

uint32_t feistel_permute_host(uint32_t i, uint32_t n, uint32_t half_bits, uint32_t key) {
  bool overflow = false;
  return feistel_permute(i, n, half_bits, key, &overflow);
}

cudaError_t gather_minibatch(const GatherArgs& a, cudaStream_t s) {
  if (a.B <= 0 || a.models < 1 || a.models > kGatherModels || a.copies < 1) return cudaErrorInvalidValue;
  int max_rows = 0;
  for (int m = 0; m < a.models; ++m) {
    if (a.dim[m] > kGatherMaxD || a.rows[m] < 1 || a.rows[m] > a.copies * a.B) return cudaErrorInvalidValue;
    max_rows = max(max_rows, a.rows[m]);
  }
  launch_pdl(gather_minibatch_kernel, dim3(grid_for(max_rows, 8 * kGatherRows, 148 * 16)), dim3(256), 0, s, a);
  return cudaGetLastError();
}

int adv_gather_blocks(long long n) {
  const long long b = (n + 255) / 256;
  return static_cast<int>(b < kAdvGatherBlocks ? (b < 1 ? 1 : b) : kAdvGatherBlocks);
}

cudaError_t adv_gather_stats(const float* adv, long long n_adv, const int* idx, long long n, float* out,
                             double* partial, unsigned int* status, cudaStream_t s) {
  if (n <= 0) return cudaErrorInvalidValue;
  adv_gather_stats_kernel<<<adv_gather_blocks(n), 256, 0, s>>>(adv, n_adv, idx, n, out, partial, status);
  return cudaGetLastError();
}

bool debug_bounds_enabled() {
#ifdef RL_DEBUG_BOUNDS
  return true;
#else
  return false;
#endif
}

int ppo_loss_blocks(int B) {
  const int groups = (B + kLossRowsPerBlock - 1) / kLossRowsPerBlock;
  return groups < kLossGridCap ? groups : kLossGridCap;
}

cudaError_t ppo_loss(const PpoLossArgs& a, cudaStream_t s) {
  if (a.A > kLossMaxA || a.B <= 0) return cudaErrorInvalidValue;
  if (a.copies < 1 || a.n0 <= 0 || a.B != a.copies * a.n0) return cudaErrorInvalidValue;
  const bool aligned = (reinterpret_cast<uintptr_t>(a.d_head) & 7) == 0 && (a.ld_dhead % 4) == 0 &&
                       (a.ld_dvalue != 8 || (reinterpret_cast<uintptr_t>(a.d_value) & 15) == 0);
  if (a.copies > 1)
    launch_pdl(ppo_loss_kernel<true>, dim3(ppo_loss_blocks(a.B)), dim3(kLossWarps * 32), 0, s, a);
  else if (a.A <= 32 && aligned)
    launch_pdl(ppo_loss_rows8_kernel, dim3(ppo_loss_blocks(a.B)), dim3(kLoss8Warps * 32), 0, s, a);
  else
    launch_pdl(ppo_loss_kernel<false>, dim3(ppo_loss_blocks(a.B)), dim3(kLossWarps * 32), 0, s, a);
  return cudaGetLastError();
}

cudaError_t reduce_segments(const ReduceSegment* segs_dev, int nseg, int total_chunks, float* send0, float* send1,
                            const unsigned int* epoch, int accumulate, cudaStream_t s) {
  if (nseg <= 0 || total_chunks <= 0) return cudaErrorInvalidValue;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int want = (total_chunks + kReduceWarps - 1) / kReduceWarps;
  const int grid = want < sms * 8 ? want : sms * 8;  // up to 64 resident warps per SM
  launch_pdl(reduce_segments_kernel, dim3(grid), dim3(kReduceWarps * 32), 0, s, segs_dev, nseg, total_chunks, send0,
             send1, epoch, accumulate);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256) rnd_intrinsic_kernel(const float* __restrict__ target, int ld_target,
                                                            const float* __restrict__ pred, int ld_pred, int rows,
                                                            int dim, const float* __restrict__ weight,
                                                            float* __restrict__ out, float* __restrict__ disc,
                                                            float gamma) {
  griddep_wait();  // launched with programmatic stream serialization (launch_pdl)
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const float w = disc ? 1.0f : *weight;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < rows; i += (gridDim.x * blockDim.x) >> 5) {
    float s = 0.f;
    for (int j = lane; j < dim; j += 32) {
      const float d = target[static_cast<size_t>(i) * ld_target + j] - pred[static_cast<size_t>(i) * ld_pred + j];
      s += d * d;
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
      const float r = sqrtf(s);
      out[i] = w * r;
      if (disc) disc[i] = gamma * disc[i] + r;
    }
  }
}

__global__ void __launch_bounds__(256) rnd_reward_scale_kernel(float* __restrict__ out, int rows,
                                                               const float* __restrict__ weight,
                                                               const float* __restrict__ std) {
  const float sd = *std;
  const float f = *weight / (sd > 0.f ? sd : 1.0f);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) out[i] *= f;
}

cudaError_t rnd_intrinsic(const float* target, int ld_target, const float* pred, int ld_pred, int rows, int dim,
                          const float* weight, float* out, float* disc, float gamma, cudaStream_t s) {
  if (rows <= 0 || dim <= 0) return cudaErrorInvalidValue;
  launch_pdl(rnd_intrinsic_kernel, dim3(grid_for(rows, 8, 148 * 16)), dim3(256), 0, s, target, ld_target, pred,
             ld_pred, rows, dim, weight, out, disc, gamma);
  return cudaGetLastError();
}

cudaError_t rnd_reward_scale(float* out, int rows, const float* weight, const float* std, cudaStream_t s) {
  if (rows <= 0) return cudaErrorInvalidValue;
  rnd_reward_scale_kernel<<<grid_for(rows, 256, 148 * 4), 256, 0, s>>>(out, rows, weight, std);
  return cudaGetLastError();
}

int mse_blocks(int rows) {
  const int groups = (rows + kMseRowsPerBlock - 1) / kMseRowsPerBlock;
  return groups < 4 * 148 ? groups : 4 * 148;
}

cudaError_t mse_grad(const MseArgs& a, cudaStream_t s) {
  if (a.A > 64 || a.rows <= 0 || a.ld_grad > 64 || a.head_cols > 64 || a.head_cols < a.A || a.ld_grad < a.A)
    return cudaErrorInvalidValue;
  launch_pdl(mse_grad_kernel, dim3(mse_blocks(a.rows)), dim3(kMseWarps * 32), 0, s, a);
  return cudaGetLastError();
}

int adam_grid(int device) {
  int sms = 148, per_sm = 1;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, adam_step_kernel, kAdamThreads, 0);
  if (per_sm < 1) per_sm = 1;
  return sms * (per_sm > 2 ? 2 : per_sm);
}

cudaError_t adam_step(const AdamArgs& a, int grid, cudaStream_t s) {
  if (a.ngroups < 1 || a.ngroups > kAdamMaxGroups) return cudaErrorInvalidValue;
  void* args[] = {const_cast<AdamArgs*>(&a)};
  return cudaLaunchCooperativeKernel(reinterpret_cast<void*>(adam_step_kernel), dim3(grid), dim3(kAdamThreads), args,
                                     0, s);
}

int colstats_chunks(long long rows) { return static_cast<int>((rows + kStatsRowsPerChunk - 1) / kStatsRowsPerChunk); }

cudaError_t colstats(const ColStatsArgs& a, cudaStream_t s) {
  dim3 grid((a.dim + 31) / 32, a.chunks);
  colstats_kernel<<<grid, dim3(32, 8), 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t norm_update(const NormUpdateArgs& a, cudaStream_t s) {
  norm_update_kernel<<<1, dim3(32, 32), 0, s>>>(a);
  return cudaGetLastError();
}

__global__ void counter_add_kernel(unsigned int* p, unsigned int delta) { *p += delta; }

cudaError_t counter_add(unsigned int* p, unsigned int delta, cudaStream_t s) {
  counter_add_kernel<<<1, 1, 0, s>>>(p, delta);
  return cudaGetLastError();
}

cudaError_t to_bf16_padded(const float* src, int rows, int cols, void* dst, int ld, cudaStream_t s) {
  to_bf16_padded_kernel<<<grid_for(static_cast<long long>(rows) * ld, 256), 256, 0, s>>>(
      src, rows, cols, static_cast<__nv_bfloat16*>(dst), ld);
  return cudaGetLastError();
}

}  // namespace rlb
