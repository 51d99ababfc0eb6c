// Counter-based N(0,1) generator for inputs generated on the device.
//
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): ten rounds of the 4x32
// Philox S-box with the published round multipliers and Weyl key increments.
// Element e of the stream keyed by `seed` takes block counter (e / 4) as the
// 64-bit low half of the counter; its four 32-bit words u0..u3 become two
// Box-Muller pairs, (u0,u1) -> elements 4b, 4b+1 and (u2,u3) -> 4b+2, 4b+3,
// with u -> (u + 1) * 2^-32 in (0, 1].  Because every element depends only on
// (seed, e), a tensor split over any number of GPUs is the same tensor.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ftb {

__host__ __device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)M0 * c[0];
    const uint64_t p1 = (uint64_t)M1 * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
    k0 += W0;
    k1 += W1;
  }
}

// Writes elements [first, first + count) of the stream to out[0 .. count).
__global__ void philox_normal_kernel(float* __restrict__ out, uint64_t seed, uint64_t first, uint64_t count) {
  const float two_pi = 6.2831853071795864769f;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t blk0 = first >> 2;
  const uint64_t blk1 = (first + count + 3) >> 2;
  for (uint64_t blk = blk0 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; blk < blk1; blk += stride) {
    uint32_t c[4] = {(uint32_t)blk, (uint32_t)(blk >> 32), 0u, 0u};
    philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
    float z[4];
#pragma unroll
    for (int pair = 0; pair < 2; ++pair) {
      const float u1 = ((float)c[2 * pair] + 1.0f) * 2.3283064365386963e-10f;
      const float u2 = ((float)c[2 * pair + 1] + 1.0f) * 2.3283064365386963e-10f;
      const float r = sqrtf(-2.0f * logf(u1));
      const float t = two_pi * u2;
      z[2 * pair] = r * cosf(t);
      z[2 * pair + 1] = r * sinf(t);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint64_t e = blk * 4 + j;
      if (e >= first && e < first + count) out[e - first] = z[j];
    }
  }
}

}  // namespace ftb
