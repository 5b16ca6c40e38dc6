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
//    address up with cudaGetSymbolAddress while that device is current and caches it together with the identity of
//    the device's current context; a call in a new context (after cudaDeviceReset, for instance) looks it up again.
//    Make the first call on a device, and the first one after its context was recreated, outside stream capture.
//  * All calls on a device share the one scratch array, and it keeps the last call's partial sums. Every partial sum
//    is written before it is read within a call, so nothing has to start at zero, but two calls whose kernels
//    overlap on the GPU (for example on two unsynchronised streams) race on the array; order such calls.
//  * Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
//  * Returns 0 (cudaSuccess) or the cudaError_t value of the failure.
#include "gae_noalloc.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "rl_kernels.cuh"

namespace {

constexpr int kMaxEnvs = RLB_GAE_NOALLOC_MAX_ENVS;
constexpr int kThreadsPerBlock = 256;  // environments per GAE block (matches the regular launcher)
constexpr int kMaxBlocks = kMaxEnvs / kThreadsPerBlock;
constexpr int kMaxDevices = 64;

// two doubles (sum, sum of squares) per 256-environment block
static __device__ __align__(256) double g_gae_scratch[2 * kMaxBlocks];

std::mutex g_lock;
void* g_scratch_addr[kMaxDevices] = {nullptr};
unsigned long long g_scratch_ctx[kMaxDevices] = {0};  // id of the context the cached address belongs to

// Unique id of the calling thread's current context (driver entry points found through the runtime, so no link
// against the driver library is needed). 0 when it cannot be determined: the address is then looked up every call.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

cudaError_t scratch_for_current_device(double** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> guard(g_lock);
  const unsigned long long ctx = current_context_id();
  if (g_scratch_addr[dev] == nullptr || ctx == 0 || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gae_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
    // read again after the lookup: cudaGetSymbolAddress makes the primary context current if none was
    g_scratch_ctx[dev] = current_context_id();
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
