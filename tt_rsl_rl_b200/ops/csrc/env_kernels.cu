// Synthetic linear-Gaussian environment step after the matmuls, one warp per environment:
//   s' = next + noise_std * eps          (eps: caller-supplied or Philox4x32-10 normals keyed by (env, element group))
//   reward = -(|s'|^2 + 0.01 |a|^2)
//   episode length + 1; terminated with probability reset_prob (a Philox uniform per env); timed out at max_len
//   state = done ? N(0, I) : s';  episode length = done ? 0 : length
//   observations: policy = state; critic = [state, |state|^2 / S, |a|^2 / A, length / max_len, 0...]
// The semantics are those of LinearGaussianVecEnv.step (tt_rsl_rl_b200/env/linear_gaussian.py), with the device's
// random streams drawn from Philox instead of the PyTorch generator.
#include "env_kernels.cuh"
#include "philox.cuh"

namespace rlb {
namespace {

constexpr uint32_t kStreamNoise = 0u;         // Philox counter word 1 offsets of the three random streams
constexpr uint32_t kStreamUniform = 1u << 30;
constexpr uint32_t kStreamReset = 2u << 30;

__device__ __forceinline__ float normal_at(uint32_t env, uint32_t elem, uint32_t stream, uint64_t step, uint64_t seed) {
  const Philox r = philox10(env, stream | (elem >> 2), static_cast<uint32_t>(step), static_cast<uint32_t>(step >> 32),
                            static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  float n0, n1, n2, n3;
  box_muller(r.c[0], r.c[1], n0, n1);
  box_muller(r.c[2], r.c[3], n2, n3);
  const int k = elem & 3;
  return k == 0 ? n0 : k == 1 ? n1 : k == 2 ? n2 : n3;
}

__global__ void __launch_bounds__(256) lg_env_step_kernel(const LgEnvArgs a) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const uint64_t step = *a.counter;
  for (int env = blockIdx.x * warps + (threadIdx.x >> 5); env < a.N; env += gridDim.x * warps) {
    const uint32_t e = static_cast<uint32_t>(env);
    const float* nx = a.next + static_cast<size_t>(env) * a.S;
    float ss = 0.f;
    float sn[8];  // S <= 256: lane holds elements lane + 32 k
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = lane + 32 * k;
      sn[k] = 0.f;
      if (j < a.S) {
        const float eps = a.noise ? a.noise[static_cast<size_t>(env) * a.S + j]
                                  : normal_at(e, static_cast<uint32_t>(j), kStreamNoise, step, a.seed);
        sn[k] = nx[j] + a.noise_std * eps;
        ss += sn[k] * sn[k];
      }
    }
    float sa = 0.f;
    for (int j = lane; j < a.A; j += 32) {
      const float v = a.actions[static_cast<size_t>(env) * a.ld_act + j];
      sa += v * v;
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, off);
      sa += __shfl_xor_sync(0xffffffffu, sa, off);
    }
    // termination draw (one uniform per env), identical on every lane
    const Philox ru = philox10(e, kStreamUniform, static_cast<uint32_t>(step), static_cast<uint32_t>(step >> 32),
                               static_cast<uint32_t>(a.seed), static_cast<uint32_t>(a.seed >> 32));
    const bool terminated = u01(ru.c[0]) < a.reset_prob;
    const long long len = a.ep_len[env] + 1;
    const bool timed_out = len >= a.max_len;
    const bool done = terminated || timed_out;
    const long long new_len = done ? 0 : len;
    // new state (reset draws N(0, I)) and its squared norm for the privileged feature
    float ns = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = lane + 32 * k;
      if (j < a.S) {
        const float v = done ? normal_at(e, static_cast<uint32_t>(j), kStreamReset, step, a.seed) : sn[k];
        a.state[static_cast<size_t>(env) * a.S + j] = v;
        a.obs_policy[static_cast<size_t>(env) * a.S + j] = v;
        if (a.obs_critic) a.obs_critic[static_cast<size_t>(env) * (a.S + a.P) + j] = v;
        ns += v * v;
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) ns += __shfl_xor_sync(0xffffffffu, ns, off);
    if (a.obs_critic && lane < a.P) {
      float f = 0.f;
      if (lane == 0) f = ns / static_cast<float>(a.S);
      if (lane == 1) f = sa / static_cast<float>(a.A);
      if (lane == 2) f = static_cast<float>(new_len) / static_cast<float>(a.max_len);
      a.obs_critic[static_cast<size_t>(env) * (a.S + a.P) + a.S + lane] = f;
    }
    if (lane == 0) {
      a.rewards[env] = -(ss + 0.01f * sa);
      a.dones[env] = done ? 1.f : 0.f;
      a.time_outs[env] = (timed_out && !terminated) ? 1.f : 0.f;
      a.ep_len[env] = new_len;
    }
  }
  // the last block to finish advances the step counter (every block read it first)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.ticket, 1u) + 1u == gridDim.x) {
      *a.counter = step + 1;
      *a.ticket = 0u;
    }
  }
}

}  // namespace

cudaError_t lg_env_step(const LgEnvArgs& a, cudaStream_t s) {
  if (a.N <= 0 || a.S <= 0 || a.S > 256 || a.A <= 0 || a.P < 0 || a.P > 32) return cudaErrorInvalidValue;
  const int warps = 8;
  long long blocks = (a.N + warps - 1) / warps;
  if (blocks > 148 * 8) blocks = 148 * 8;
  lg_env_step_kernel<<<static_cast<int>(blocks), warps * 32, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace rlb
