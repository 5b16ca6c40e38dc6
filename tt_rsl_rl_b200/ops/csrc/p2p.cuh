// Peer-to-peer collectives over mapped peer memory (CUDA IPC), with bounded flag waits.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rlb {

constexpr int kMaxWorld = 8;

struct P2PArgs {
  int world, rank;
  const void* peer_buf[kMaxWorld];      // every rank's symmetric buffer (index = rank; own buffer at [rank])
  unsigned int* peer_flags[kMaxWorld];  // every rank's flag array ([world] uint32 each)
  unsigned int* epoch;                  // this rank's device epoch counter of the channel
  uint64_t timeout_ns;
  unsigned int* status;
};

// out[i] = sum over ranks, in rank order, of peer_buf[r][i] (double); bit-identical on every rank.
cudaError_t p2p_allreduce_f64(const P2PArgs& a, double* out, long long n, cudaStream_t s);
// dst[i] = peer_buf[root][i] (float) on every rank.
cudaError_t p2p_broadcast_f32(const P2PArgs& a, int root, float* dst, long long n, cudaStream_t s);

}  // namespace rlb
