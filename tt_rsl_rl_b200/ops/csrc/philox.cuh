// Philox4x32-10 counter-based random numbers and the Box-Muller transform, shared by the policy sampler and the
// synthetic environment kernel.
#pragma once

#include <stdint.h>

namespace rlb {

// ---------------------------------------------------------------------------------------------------------------
// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011). Multipliers and Weyl key increments are the published Philox4x32 constants.
// ---------------------------------------------------------------------------------------------------------------
struct Philox {
  uint32_t c[4];
};
__device__ __forceinline__ Philox philox10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                           uint32_t k1) {
  Philox r{{c0, c1, c2, c3}};
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, r.c[0]);
    const uint32_t lo0 = 0xD2511F53u * r.c[0];
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, r.c[2]);
    const uint32_t lo1 = 0xCD9E8D57u * r.c[2];
    r = Philox{{hi1 ^ r.c[1] ^ k0, lo1, hi0 ^ r.c[3] ^ k1, lo0}};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return r;
}
// uint32 -> uniform in (0, 1)
__device__ __forceinline__ float u01(uint32_t x) { return (static_cast<float>(x) + 0.5f) * 2.3283064365386963e-10f; }
// Box-Muller transform of two uniforms into two standard normals.
__device__ __forceinline__ void box_muller(uint32_t a, uint32_t b, float& n0, float& n1) {
  const float r = sqrtf(-2.0f * logf(u01(a)));
  float s, c;
  sincospif(2.0f * u01(b), &s, &c);
  n0 = r * c;
  n1 = r * s;
}


}  // namespace rlb
