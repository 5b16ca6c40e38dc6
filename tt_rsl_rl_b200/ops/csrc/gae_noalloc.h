// C interface of the allocation-free GAE entry point (implemented in gae_noalloc.cu). This entry point has no
// counterpart in the reference.
//
// For callers that must not allocate device memory while they run (a C or C++ learner inside a control process that
// reserves all of its memory at start-up, or host code without a caching allocator): the caller passes its device
// buffers, and the only scratch space, per-block partial sums of the advantage statistics, is a fixed device array
// inside the library (64 KiB per GPU that loads it, held until the process exits).
//
//   rewards, dones, values, returns, advantages: float32 [T * N], step-major (row t * N + n); dones as 0.0 / 1.0
//   last_values: float32 [N], the value of the observation after the last step
//   normalize != 0: advantages = (A - mean) / (unbiased std + 1e-8) over all T * N entries; otherwise A = R - V
//
// Rules: N <= RLB_GAE_NOALLOC_MAX_ENVS (larger N is rejected with cudaErrorInvalidValue before anything runs); the
// first call on a device (and the first call after that device's context was recreated, e.g. after
// cudaDeviceReset) looks up the scratch array's device address, so make it outside stream capture; calls whose
// kernels overlap on one GPU race on the shared scratch array and must be ordered. Nothing allocates.
// Returns 0 (cudaSuccess) or a cudaError_t value.
#pragma once

#include <cuda_runtime.h>

#define RLB_GAE_NOALLOC_MAX_ENVS (1 << 20)

#ifdef __cplusplus
extern "C" {
#endif

int rlb_gae_advantages_noalloc(const float* rewards, const float* dones, const float* values, const float* last_values,
                               float* returns, float* advantages, int T, int N, float gamma, float lam, int normalize,
                               cudaStream_t stream);

#ifdef __cplusplus
}
#endif
