// Fused GEMM / conv epilogue shared by the SIMT and tensor-core kernels.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

#include "flags.h"

namespace ftb {

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device
// (the attribute belongs to the device's context); `done` holds one bit per
// device and may be shared by threads.  Returns the CUDA status it saw.
template <typename Kernel>
inline cudaError_t smem_limit_once(Kernel kernel, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const uint64_t bit = 1ull << dev;
  if (done.load() & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  done.fetch_or(bit);
  return cudaSuccess;
}

// The CUDA status of this thread's most recent launch check.  A launcher that
// returns -1 after its own cudaGetLastError() has consumed (and cleared) the
// error keeps it here, so the caller's message can still name it.
inline cudaError_t& launch_error_slot() {
  static thread_local cudaError_t e = cudaSuccess;
  return e;
}
inline int note_launch(cudaError_t e) {
  launch_error_slot() = e;
  return e == cudaSuccess ? 0 : -1;
}
// The error behind the last failed launch: the kept status, else whatever
// the runtime still holds.
inline cudaError_t take_launch_error() {
  const cudaError_t e = launch_error_slot();
  launch_error_slot() = cudaSuccess;
  return e != cudaSuccess ? e : cudaGetLastError();
}

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
