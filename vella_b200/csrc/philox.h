// Philox-4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011), usable from host and device code.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define VELLA_HD __host__ __device__ __forceinline__
#else
#define VELLA_HD inline
#endif

namespace vella {

struct U4 {
  uint32_t x, y, z, w;
};

VELLA_HD void mulhilo32(uint32_t a, uint32_t b, uint32_t* hi, uint32_t* lo) {
  const uint64_t p = static_cast<uint64_t>(a) * b;
  *hi = static_cast<uint32_t>(p >> 32);
  *lo = static_cast<uint32_t>(p);
}

// 10 rounds of Philox-4x32 on counter c with key (k0, k1).
VELLA_HD U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(M0, c.x, &hi0, &lo0);
    mulhilo32(M1, c.z, &hi1, &lo1);
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += W0;
    k1 += W1;
  }
  return c;
}

// Uniform in [0, 1) from the top 24 bits.
VELLA_HD float u01(uint32_t v) { return static_cast<float>(v >> 8) * (1.0f / 16777216.0f); }

}  // namespace vella
