// Flags shared by the host engine and the device kernels.
#pragma once

#include <cstdint>

namespace ftb {

// Epilogue applied to the accumulator of a GEMM / conv, in this order:
//   [bias (first: accumulator starts at the bias / last: added after the sum)]
//   [relu] [+ residual] [relu]
// Every step is a separately rounded fp32 operation, the order the
// reference's un-fused ADD / RELU loops apply them in.
enum EpiFlags : uint32_t {
  EPI_BIAS_FIRST = 1u << 0,
  EPI_BIAS_LAST = 1u << 1,
  EPI_RELU_PRE = 1u << 2,
  EPI_RESIDUAL = 1u << 3,
  EPI_RELU_POST = 1u << 4,
  EPI_BIAS_ROWS = 1u << 5,  // bias is [M,N] instead of [N]
};

}  // namespace ftb
