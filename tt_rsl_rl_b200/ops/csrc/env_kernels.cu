// Synthetic linear-Gaussian environment step in one launch, one warp per environment:
//   s' = A s + B a + noise_std * eps     (the transition matrices in shared memory; eps: caller-supplied or Philox)
//   reward = -(|s'|^2 + 0.01 |a|^2)
//   episode length + 1; terminated with probability reset_prob (a Philox uniform per env); timed out at max_len
//   state = done ? N(0, I) : s';  episode length = done ? 0 : length
//   observations: policy = state; critic = [state, |state|^2 / S, |a|^2 / A, length / max_len, 0...]
// Lane l owns state elements 4 l .. 4 l + 3 (S <= 128, S % 4 == 0): it accumulates their rows of the matrix-vector
// products from float4 rows of A^T and B^T (conflict-free shared-memory loads, the vector element broadcast), and one
// Philox4x32-10 block (Salmon et al., SC'11) per lane and stream gives its four normals (Box-Muller on two pairs).
// The semantics are those of LinearGaussianVecEnv.step (tt_rsl_rl_b200/env/linear_gaussian.py), with the device's
// random streams drawn from Philox instead of the PyTorch generator.
#include "env_kernels.cuh"
#include "philox.cuh"

namespace rlb {
namespace {

constexpr uint32_t kStreamNoise = 0u;         // Philox counter word 1 offsets of the three random streams
constexpr uint32_t kStreamUniform = 1u << 30;
constexpr uint32_t kStreamReset = 2u << 30;

// Normals of state elements 4 q .. 4 q + 3 of environment env: one Philox block keyed by (env, stream | q, step).
__device__ __forceinline__ float4 normals4(uint32_t env, uint32_t q, uint32_t stream, uint64_t step, uint64_t seed) {
  const Philox r = philox10(env, stream | q, static_cast<uint32_t>(step), static_cast<uint32_t>(step >> 32),
                            static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  float4 n;
  box_muller(r.c[0], r.c[1], n.x, n.y);
  box_muller(r.c[2], r.c[3], n.z, n.w);
  return n;
}

constexpr int kEnvWarps = 8;

__global__ void __launch_bounds__(kEnvWarps * 32) lg_env_step_kernel(const LgEnvArgs a) {
  extern __shared__ float4 env_smem4[];
  float* smem = reinterpret_cast<float*>(env_smem4);
  float* At = smem;                           // [S, S]: At[i * S + j] = A[j][i]
  float* Bt = At + a.S * a.S;                 // [A, S]
  float* vec = Bt + a.A * a.S;                // per warp: the state row then the action row
  const int vec_stride = a.S + ((a.A + 3) & ~3);  // floats per warp slot: a multiple of 4 (16-byte float4 stores)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int k = threadIdx.x; k < a.S * a.S; k += blockDim.x) At[k] = a.At[k];
  for (int k = threadIdx.x; k < a.A * a.S; k += blockDim.x) Bt[k] = a.Bt[k];
  __syncthreads();
  float* wv = vec + warp * vec_stride;
  const int S4 = a.S / 4;
  const bool own = lane < S4;
  const uint64_t step = *a.counter;
  for (int env = blockIdx.x * kEnvWarps + warp; env < a.N; env += gridDim.x * kEnvWarps) {
    const uint32_t e = static_cast<uint32_t>(env);
    const float4* s_row = reinterpret_cast<const float4*>(a.state + static_cast<size_t>(env) * a.S);
    float4 s4 = own ? s_row[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (own) reinterpret_cast<float4*>(wv)[lane] = s4;
    float sa = 0.f;
    for (int j = lane; j < a.A; j += 32) {
      const float v = a.actions[static_cast<size_t>(env) * a.ld_act + j];
      wv[a.S + j] = v;
      sa += v * v;
    }
    __syncwarp();
    // s' = A s + B a for this lane's four elements
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (own) {
      for (int i = 0; i < a.S; ++i) {
        const float x = wv[i];
        const float4 m = reinterpret_cast<const float4*>(At + i * a.S)[lane];
        acc.x = fmaf(x, m.x, acc.x);
        acc.y = fmaf(x, m.y, acc.y);
        acc.z = fmaf(x, m.z, acc.z);
        acc.w = fmaf(x, m.w, acc.w);
      }
      for (int i = 0; i < a.A; ++i) {
        const float x = wv[a.S + i];
        const float4 m = reinterpret_cast<const float4*>(Bt + i * a.S)[lane];
        acc.x = fmaf(x, m.x, acc.x);
        acc.y = fmaf(x, m.y, acc.y);
        acc.z = fmaf(x, m.z, acc.z);
        acc.w = fmaf(x, m.w, acc.w);
      }
      const float4 eps = a.noise ? reinterpret_cast<const float4*>(a.noise + static_cast<size_t>(env) * a.S)[lane]
                                 : normals4(e, static_cast<uint32_t>(lane), kStreamNoise, step, a.seed);
      acc.x += a.noise_std * eps.x;
      acc.y += a.noise_std * eps.y;
      acc.z += a.noise_std * eps.z;
      acc.w += a.noise_std * eps.w;
    }
    float ss = acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
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
    if (own) {
      const float4 v = done ? normals4(e, static_cast<uint32_t>(lane), kStreamReset, step, a.seed) : acc;
      reinterpret_cast<float4*>(a.state + static_cast<size_t>(env) * a.S)[lane] = v;
      reinterpret_cast<float4*>(a.obs_policy + static_cast<size_t>(env) * a.S)[lane] = v;
      if (a.obs_critic) {
        float* c = a.obs_critic + static_cast<size_t>(env) * (a.S + a.P) + 4 * lane;
        c[0] = v.x;
        c[1] = v.y;
        c[2] = v.z;
        c[3] = v.w;
      }
      ns = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
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
    __syncwarp();  // the warp's vector buffer is rewritten for its next environment
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

size_t lg_env_smem_bytes(int S, int A) {
  return sizeof(float) * (static_cast<size_t>(S) * S + static_cast<size_t>(A) * S + kEnvWarps * (S + ((A + 3) & ~3)));
}

cudaError_t lg_env_step(const LgEnvArgs& a, cudaStream_t s) {
  if (a.N <= 0 || a.S <= 0 || a.S > 128 || (a.S % 4) != 0 || a.A <= 0 || a.A > 64 || a.P < 0 || a.P > 32)
    return cudaErrorInvalidValue;
  const size_t smem = lg_env_smem_bytes(a.S, a.A);
  static size_t configured = 0;
  if (smem > 48 * 1024 && smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(lg_env_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  long long blocks = (a.N + kEnvWarps - 1) / kEnvWarps;
  if (blocks > 148 * 4) blocks = 148 * 4;
  lg_env_step_kernel<<<static_cast<int>(blocks), kEnvWarps * 32, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace rlb
