// Fused step of the synthetic linear-Gaussian environment (transition, noise, reward, resets, observations).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rlb {

struct LgEnvArgs {
  int N, S, A, P;          // environments, state dim, action dim, privileged critic features (critic width S + P)
  const float* At;         // [S, S] A^T (row-major: At[i * S + j] = A[j][i])
  const float* Bt;         // [A, S] B^T
  float* state;            // [N, S] in: s; out: the new state (reset where done). S <= 128, S % 4 == 0, A <= 64
  const float* actions;    // [N, A] row pitch ld_act
  int ld_act;
  const float* noise;      // optional [N, S] process noise supplied by the caller (else Philox normals)
  float noise_std, reset_prob;
  long long max_len;
  long long* ep_len;       // [N] in/out
  float* rewards;          // [N] -(|s'|^2 + 0.01 |a|^2)
  float* dones;            // [N]
  float* time_outs;        // [N]
  float* obs_policy;       // [N, S]
  float* obs_critic;       // [N, S + P] or null
  uint64_t seed;
  uint64_t* counter;       // Philox step counter, advanced once per launch by the last block to finish
  unsigned int* ticket;
};

cudaError_t lg_env_step(const LgEnvArgs& a, cudaStream_t s);
size_t lg_env_smem_bytes(int S, int A);

}  // namespace rlb
