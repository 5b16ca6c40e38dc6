// Peer-to-peer collectives over NVLink / NVSwitch for the data-parallel engine.
//
// Buffers are plain cudaMalloc allocations shared between the ranks of one node through CUDA IPC handles; each
// rank maps every peer's buffer once, so kernels read peer memory with ordinary loads (no TMA on peer memory).
// Synchronisation uses monotonically increasing epochs: a rank publishes `epoch` into slot `rank` of every peer's
// flag array (st.release.sys) and waits (ld.acquire.sys, bounded by %globaltimer) until every slot of its own
// array has reached `epoch`. On timeout the kernel records the failing peer in the status word and returns.
#include <cuda_runtime.h>
#include <stdint.h>

#include "p2p.cuh"
#include "sm100_primitives.cuh"

namespace rlb {
namespace {

__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Publish this rank's epoch to every peer and wait for all peers. Called by one thread. Returns false on timeout.
__device__ bool flag_barrier(const P2PArgs& a, unsigned int epoch) {
  __threadfence_system();
  for (int r = 0; r < a.world; ++r) st_release_sys_u32(a.peer_flags[r] + a.rank, epoch);
  const uint64_t t0 = globaltimer_ns();
  const unsigned int* mine = a.peer_flags[a.rank];
  for (int r = 0; r < a.world; ++r) {
    while (static_cast<int>(ld_acquire_sys_u32(mine + r) - epoch) < 0) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        report_error(a.status, kTimeoutPeerFlag, 100 + r);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// out[i] = sum over ranks (rank order) of peer_src[r][i]; single block (small vectors: normaliser moments).
__global__ void allreduce_f64_kernel(const P2PArgs a, double* out, long long n) {
  __shared__ int ok;
  __shared__ unsigned int epoch_s;
  if (threadIdx.x == 0) {
    epoch_s = *a.epoch + 1u;
    ok = flag_barrier(a, epoch_s) ? 1 : 0;
  }
  __syncthreads();
  if (ok) {
    for (long long i = threadIdx.x; i < n; i += blockDim.x) {
      double s = 0.0;
      for (int r = 0; r < a.world; ++r) s += static_cast<const double*>(a.peer_buf[r])[i];
      out[i] = s;
    }
  }
  __syncthreads();
  // second barrier: no rank may overwrite its buffer for the next exchange before every peer has read it
  if (threadIdx.x == 0 && ok) {
    if (!flag_barrier(a, epoch_s + 1u)) ok = 0;
    *a.epoch = epoch_s + 1u;
  } else if (threadIdx.x == 0) {
    *a.epoch = epoch_s + 1u;
  }
}

// dst[i] = peer_buf[root][i] for all ranks (including the root), bracketed by two flag barriers.
__global__ void broadcast_f32_kernel(const P2PArgs a, int root, float* dst, long long n) {
  __shared__ int ok;
  __shared__ unsigned int epoch_s;
  if (threadIdx.x == 0) {
    epoch_s = *a.epoch + 1u;
    ok = flag_barrier(a, epoch_s) ? 1 : 0;
  }
  __syncthreads();
  if (ok) {
    const float* src = static_cast<const float*>(a.peer_buf[root]);
    for (long long i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (ok) flag_barrier(a, epoch_s + 1u);
    *a.epoch = epoch_s + 1u;
  }
}

}  // namespace

cudaError_t p2p_allreduce_f64(const P2PArgs& a, double* out, long long n, cudaStream_t s) {
  allreduce_f64_kernel<<<1, 256, 0, s>>>(a, out, n);
  return cudaGetLastError();
}

cudaError_t p2p_broadcast_f32(const P2PArgs& a, int root, float* dst, long long n, cudaStream_t s) {
  broadcast_f32_kernel<<<1, 1024, 0, s>>>(a, root, dst, n);
  return cudaGetLastError();
}

}  // namespace rlb
