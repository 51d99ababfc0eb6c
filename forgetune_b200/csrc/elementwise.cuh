// Elementwise kernels for the nodes that stay un-fused: ADD / MUL with the
// reference's three broadcast forms (src/codegen.cpp:870-958), RELU, SIGMOID,
// TANH and plain copies (FLATTEN that is a graph output, OUTPUT, identity and
// constant outputs, src/codegen.cpp:860-869, 960-993).  Grid-stride loops over
// the flat index; each element is one separately rounded fp32 operation, so
// ADD / MUL / RELU / copies are bit-identical to the reference loops.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "epilogue.cuh"

namespace ftb {

enum EwOp : int { EW_ADD = 0, EW_MUL = 1, EW_RELU = 2, EW_SIGMOID = 3, EW_TANH = 4, EW_COPY = 5 };

// Broadcast form of the second operand of ADD / MUL.
enum EwBcast : int { BC_SAME = 0, BC_ROW = 1, BC_CHANNEL = 2 };

template <int OP, int BC>
__global__ void ew_binary_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y,
                                 int64_t n, int64_t row_len, int64_t channels) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float bv;
    if constexpr (BC == BC_SAME) {
      bv = b[i];
    } else if constexpr (BC == BC_ROW) {
      bv = b[i % row_len];
    } else {
      bv = b[(i / row_len) % channels];
    }
    y[i] = (OP == EW_ADD) ? __fadd_rn(a[i], bv) : __fmul_rn(a[i], bv);
  }
}

template <int OP>
__global__ void ew_unary_kernel(const float* __restrict__ a, float* __restrict__ y, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = a[i];
    float r;
    if constexpr (OP == EW_RELU) {
      r = relu_keep_nan(v);
    } else if constexpr (OP == EW_SIGMOID) {
      r = 1.0f / (1.0f + expf(-v));
    } else if constexpr (OP == EW_TANH) {
      r = tanhf(v);
    } else {
      r = v;
    }
    y[i] = r;
  }
}

// float4 copy for 16-byte aligned, multiple-of-4 element counts
__global__ void copy4_kernel(const float4* __restrict__ a, float4* __restrict__ y, int64_t n4) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) y[i] = a[i];
}

}  // namespace ftb
