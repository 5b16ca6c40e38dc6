// No-allocation entry point for GAE returns + advantage normalisation. This entry point has no counterpart in the
// reference: upstream computes returns with PyTorch tensor operations that allocate as they go.
//
// Who it is for: callers that must not allocate device memory while they run. Examples are a C or C++ learner linked
// into a robot's control process, which reserves all of its memory at start-up and may not call cudaMalloc (or grow
// any allocator) inside its control loop, and host code without PyTorch that therefore has no caching allocator to
// borrow scratch space from. Such a caller owns its input and output buffers and passes them in; the only scratch
// space this computation needs, two per-block partial sums for the advantage mean and variance, lives in a fixed
// device array defined in this file instead of a buffer the caller would have to allocate.
//
// Rules for callers:
//  * At most kMaxEnvs (1,048,576) environments per call; larger N is rejected with cudaErrorInvalidValue before
//    anything is launched. T may be any positive value.
//  * The scratch array is a file-scope __device__ variable: every GPU that loads this library holds its 64 KiB until
//    the process exits. Its host-side name is not a device address, so the first call on each device looks the
//    address up with cudaGetSymbolAddress while that device is current and caches it. Make that first call outside
//    any CUDA stream capture.
//  * All calls on a device share the one scratch array, and it keeps the last call's partial sums. Every partial sum
//    is written before it is read within a call, so nothing has to start at zero, but two calls whose kernels
//    overlap on the GPU (for example on two unsynchronised streams) race on the array; order such calls.
//  * Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
//  * Returns 0 (cudaSuccess) or the cudaError_t value of the failure.
#include <cuda_runtime.h>

#include <mutex>

#include "rl_kernels.cuh"

namespace {

constexpr int kMaxEnvs = 1 << 20;
constexpr int kThreadsPerBlock = 256;  // environments per GAE block (matches the regular launcher)
constexpr int kMaxBlocks = kMaxEnvs / kThreadsPerBlock;
constexpr int kMaxDevices = 64;

// two doubles (sum, sum of squares) per 256-environment block
static __device__ __align__(256) double g_gae_scratch[2 * kMaxBlocks];

std::mutex g_lock;
void* g_scratch_addr[kMaxDevices] = {nullptr};

cudaError_t scratch_for_current_device(double** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> guard(g_lock);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gae_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = static_cast<double*>(g_scratch_addr[dev]);
  return cudaSuccess;
}

}  // namespace

extern "C" int rlb_gae_advantages_noalloc(const float* rewards, const float* dones, const float* values,
                                          const float* last_values, float* returns, float* advantages, int T, int N,
                                          float gamma, float lam, int normalize, cudaStream_t stream) {
  if (T <= 0 || N <= 0 || N > kMaxEnvs) return static_cast<int>(cudaErrorInvalidValue);
  if (!rewards || !dones || !values || !last_values || !returns || !advantages)
    return static_cast<int>(cudaErrorInvalidValue);
  if (rlb::gae_blocks(N) > kMaxBlocks) return static_cast<int>(cudaErrorInvalidValue);
  double* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  rlb::GaeArgs a{rewards, dones, values, last_values, returns, advantages, T, N, gamma, lam, scratch};
  e = rlb::gae(a, stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  const long long total = static_cast<long long>(T) * N;
  if (normalize && total > 1) {
    e = rlb::adv_normalize(advantages, total, scratch, rlb::gae_blocks(N), stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return static_cast<int>(cudaSuccess);
}
