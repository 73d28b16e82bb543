// Counter-based dropout bits shared by the fused kernels that regenerate a
// dropout mask in their backward instead of storing it.
#pragma once

#include "common.cuh"

namespace affb {

// Dropout bits: Philox-4x32-10 (Salmon et al., "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011), key = (seed, a fixed word), counter = the
// element index / 4; the 4 output words belong to elements 4i .. 4i+3.  Each
// seed gives an independent pseudo-random stream (a keyed bijection of 10
// rounds), not a re-indexing of one pattern.
__host__ __device__ __forceinline__ void philox4x32_10(uint32_t k0, uint32_t k1, uint32_t c[4]) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)M0 * c[0], p1 = (uint64_t)M1 * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += W0; k1 += W1;
  }
}

constexpr uint32_t DROP_KEY1 = 0x6C62272Eu;

// The random words of elements e .. e+VEC-1.
template <int VEC>
__host__ __device__ __forceinline__ void drop_words(uint32_t seed, uint64_t e, uint32_t* w) {
  if (VEC == 4 && (e & 3) == 0) {
    uint32_t c[4] = {(uint32_t)(e >> 2), (uint32_t)(e >> 34), 0u, 0u};
    philox4x32_10(seed, DROP_KEY1, c);
    for (int k = 0; k < VEC; ++k) w[k] = c[k];
  } else {
    for (int k = 0; k < VEC; ++k) {
      const uint64_t ek = e + k;
      uint32_t c[4] = {(uint32_t)(ek >> 2), (uint32_t)(ek >> 34), 0u, 0u};
      philox4x32_10(seed, DROP_KEY1, c);
      w[k] = c[ek & 3];
    }
  }
}

// Keep an element when its word is >= this threshold (0: no dropout).
__host__ __device__ inline uint32_t drop_threshold(float p) {
  if (p <= 0.f) return 0u;
  const double t = (double)p * 4294967296.0;
  return t >= 4294967295.0 ? 4294967295u : (uint32_t)t;
}

}  // namespace affb
