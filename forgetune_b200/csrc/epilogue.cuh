// Fused GEMM / conv epilogue shared by the SIMT and tensor-core kernels.
#pragma once

#include <cstdint>

#include "flags.h"

namespace ftb {

// NaN-keeping ReLU, the reference's (std::isnan(v) || v > 0.0f) ? v : 0.0f
// (src/codegen.cpp:394, 840); fmaxf would turn NaN into 0.
__device__ __forceinline__ float relu_keep_nan(float v) { return (v != v || v > 0.0f) ? v : 0.0f; }

__device__ __forceinline__ float apply_epilogue(float acc, uint32_t epi, const float* __restrict__ bias,
                                                const float* __restrict__ res, int64_t m, int64_t n,
                                                int64_t N) {
  float v = acc;
  if (epi & EPI_BIAS_LAST) v = __fadd_rn(v, (epi & EPI_BIAS_ROWS) ? bias[m * N + n] : bias[n]);
  if (epi & EPI_RELU_PRE) v = relu_keep_nan(v);
  if (epi & EPI_RESIDUAL) v = __fadd_rn(v, res[m * N + n]);
  if (epi & EPI_RELU_POST) v = relu_keep_nan(v);
  return v;
}

}  // namespace ftb
