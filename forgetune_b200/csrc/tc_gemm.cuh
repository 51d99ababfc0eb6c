// Tensor-core (tcgen05 / TMEM) 3xTF32 GEMM for large dense layers.
#pragma once

#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#include "epilogue.cuh"

namespace ftb {

struct TcWeights {
  const float* hi = nullptr;  // W^T [N, Kp], tf32-rounded
  const float* lo = nullptr;  // W^T - hi
  int64_t Kp = 0;
};

struct TcArgs {
  const float* A;
  const float* w_hi;
  const float* w_lo;
  const float* bias;
  const float* res;
  float* Y;
  int64_t M, N, K, Kp;
  uint32_t epi;
};

inline bool tc_gemm_supported(int64_t K, int64_t N) {
  (void)K;
  (void)N;
  return false;
}

inline int64_t tc_padded_k(int64_t K) { return (K + 31) / 32 * 32; }

inline bool tc_gemm_profitable(int64_t M, int64_t K, int64_t N) {
  (void)M;
  (void)K;
  (void)N;
  return false;
}

// round-to-nearest (ties away) to the 10-bit tf32 mantissa, on the host
inline float tf32_round_host(float v) {
  uint32_t u;
  std::memcpy(&u, &v, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

inline int launch_tc_gemm(const TcArgs& t, int sm_count, cudaStream_t s) {
  (void)t;
  (void)sm_count;
  (void)s;
  return -1;
}

}  // namespace ftb
