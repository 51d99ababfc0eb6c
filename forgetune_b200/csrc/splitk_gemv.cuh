// Split-K GEMM for a handful of rows (M <= 16), the batch-1 latency path.
//
//   y[m, n] = epi( sum_k x[m, k] W[k, n] ),   W [K, N] row-major
//
// A single row of the tiny MLP's first layer is 200 K multiply-adds over an
// 800 KB weight: the time is the latency of streaming W, not arithmetic.  The
// grid is (column blocks of 64) x (KS slices of K); each CTA's eight warps
// stride over the k of its slice, every lane owning two columns, so each
// warp-wide load is a 128-byte row segment of W and many loads are in flight.
// The eight warp partials are summed in shared memory in warp order and
// written to a workspace slot [ks][m][n]; the last CTA of a column block to
// finish (an integer ticket) sums the KS slots in ks order, applies the
// epilogue and resets the ticket.  No floating-point atomics: the result does
// not depend on which CTA finishes last, so runs are bitwise reproducible.
//
// Workspace: KS * MMAX * N floats of partial sums plus one ticket per column
// block, which must be zero before the first launch (the last CTA leaves it
// zero again).
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

#include "epilogue.cuh"

namespace ftb {

constexpr int kSkCols = 64;     // columns per CTA (two per lane)
constexpr int kSkWarps = 8;
constexpr int kSkMaxKc = 512;   // k per slice, bounds the shared x chunk
constexpr int kSkMaxSlices = 64;

struct SplitKArgs {
  const float* A;     // [M, K]
  const float* B;     // [K, N]
  const float* bias;
  const float* res;
  float* Y;           // [M, N]
  float* part;        // [KS][MMAX][N]
  unsigned* tickets;  // [ceil(N / 64)]
  int M, N, K, kc, ks_count;
  uint32_t epi;
};

template <int MMAX>
__global__ void __launch_bounds__(kSkWarps * 32) splitk_gemv_kernel(SplitKArgs p) {
  extern __shared__ float sk_smem[];
  float* xs = sk_smem;                      // [MMAX][kc]
  float* red = sk_smem + MMAX * p.kc;       // [warps][MMAX][64]
  __shared__ unsigned s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.x, ks = blockIdx.y;
  const int n0 = cb * kSkCols;
  const int k0 = ks * p.kc;
  const int k1 = min(p.K, k0 + p.kc);
  const int kn = max(0, k1 - k0);

  for (int i = threadIdx.x; i < MMAX * p.kc; i += blockDim.x) {
    const int m = i / p.kc, kk = i - m * p.kc;
    xs[i] = (m < p.M && kk < kn) ? p.A[(int64_t)m * p.K + k0 + kk] : 0.0f;
  }
  __syncthreads();

  const int c0 = n0 + lane, c1 = n0 + 32 + lane;
  const bool v0 = c0 < p.N, v1 = c1 < p.N;
  float acc0[MMAX], acc1[MMAX];
#pragma unroll
  for (int m = 0; m < MMAX; ++m) acc0[m] = acc1[m] = 0.0f;
  const float* wcol = p.B + (int64_t)k0 * p.N;
  int kk = warp;
  // four k rows per iteration: eight independent loads per lane in flight
  for (; kk + 3 * kSkWarps < kn; kk += 4 * kSkWarps) {
    float w0[4], w1[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float* row = wcol + (int64_t)(kk + u * kSkWarps) * p.N;
      w0[u] = v0 ? __ldg(row + c0) : 0.0f;
      w1[u] = v1 ? __ldg(row + c1) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int m = 0; m < MMAX; ++m) {
        const float xv = xs[m * p.kc + kk + u * kSkWarps];
        acc0[m] = fmaf(xv, w0[u], acc0[m]);
        acc1[m] = fmaf(xv, w1[u], acc1[m]);
      }
    }
  }
  for (; kk < kn; kk += kSkWarps) {
    const float* row = wcol + (int64_t)kk * p.N;
    const float w0 = v0 ? __ldg(row + c0) : 0.0f;
    const float w1 = v1 ? __ldg(row + c1) : 0.0f;
#pragma unroll
    for (int m = 0; m < MMAX; ++m) {
      const float xv = xs[m * p.kc + kk];
      acc0[m] = fmaf(xv, w0, acc0[m]);
      acc1[m] = fmaf(xv, w1, acc1[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < MMAX; ++m) {
    red[(warp * MMAX + m) * kSkCols + lane] = acc0[m];
    red[(warp * MMAX + m) * kSkCols + 32 + lane] = acc1[m];
  }
  __syncthreads();
  // warp partials summed in warp order; one slot of the workspace per slice
  for (int i = threadIdx.x; i < MMAX * kSkCols; i += blockDim.x) {
    const int m = i / kSkCols, c = i - m * kSkCols;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kSkWarps; ++w) s += red[(w * MMAX + m) * kSkCols + c];
    if (m < p.M && n0 + c < p.N) p.part[((int64_t)ks * MMAX + m) * p.N + n0 + c] = s;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&p.tickets[cb], 1u) == (unsigned)(p.ks_count - 1)) ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < MMAX * kSkCols; i += blockDim.x) {
    const int m = i / kSkCols, c = i - m * kSkCols;
    const int n = n0 + c;
    if (m >= p.M || n >= p.N) continue;
    float s = 0.0f;
    for (int j = 0; j < p.ks_count; ++j) s += __ldcg(p.part + ((int64_t)j * MMAX + m) * p.N + n);
    uint32_t epi = p.epi;
    if (epi & EPI_BIAS_FIRST) epi = (epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
    p.Y[(int64_t)m * p.N + n] = apply_epilogue(s, epi, p.bias, p.res, m, n, p.N);
  }
  if (threadIdx.x == 0) p.tickets[cb] = 0u;  // ready for the next launch
}

// Slices of K: enough CTAs to cover the GPU about twice, at most 512 k per
// slice (the shared x chunk), at least 16 k per slice.
inline void splitk_shape(int64_t K, int64_t N, int sm_count, int* ks_count, int* kc) {
  const int64_t cbs = (N + kSkCols - 1) / kSkCols;
  int64_t ks = (2 * (int64_t)sm_count + cbs - 1) / cbs;
  ks = std::max<int64_t>(ks, (K + kSkMaxKc - 1) / kSkMaxKc);
  ks = std::min<int64_t>(ks, std::max<int64_t>(1, K / 16));
  ks = std::min<int64_t>(ks, kSkMaxSlices);
  int64_t c = (K + ks - 1) / ks;
  c = (c + 7) / 8 * 8;
  c = std::min<int64_t>(c, kSkMaxKc);
  *kc = (int)c;
  *ks_count = (int)((K + c - 1) / c);
}

inline size_t splitk_part_floats(int64_t K, int64_t N, int sm_count) {
  int ks, kc;
  splitk_shape(K, N, sm_count, &ks, &kc);
  return (size_t)ks * 16 * (size_t)N;
}

// Launches the split-K kernel; the caller provides `part` (at least
// splitk_part_floats floats) and zeroed `tickets` (ceil(N/64) entries).
// Returns 0 once launched, 1 when M is outside 1..16 (nothing launched), -1 on
// a CUDA error, whose status goes to *err (the launch check has already
// consumed it, so cudaGetLastError() would no longer report it).
inline int launch_splitk(SplitKArgs a, int sm_count, cudaStream_t s, cudaError_t* err) {
  *err = cudaSuccess;
  if (a.M <= 0 || a.M > 16) return 1;
  int ks, kc;
  splitk_shape(a.K, a.N, sm_count, &ks, &kc);
  a.kc = kc;
  a.ks_count = ks;
  const int mmax = a.M <= 8 ? 8 : 16;
  const size_t smem = (size_t)mmax * kc * 4 + (size_t)kSkWarps * mmax * kSkCols * 4;
  dim3 grid((unsigned)((a.N + kSkCols - 1) / kSkCols), (unsigned)ks);
  // the shared-memory limit is per device context: set once per device
  static std::atomic<uint64_t> attr8{0}, attr16{0};
  if (mmax == 8) {
    *err = smem_limit_once(splitk_gemv_kernel<8>, 96 * 1024, attr8);
    if (*err != cudaSuccess) return -1;
    splitk_gemv_kernel<8><<<grid, kSkWarps * 32, smem, s>>>(a);
  } else {
    *err = smem_limit_once(splitk_gemv_kernel<16>, 96 * 1024, attr16);
    if (*err != cudaSuccess) return -1;
    splitk_gemv_kernel<16><<<grid, kSkWarps * 32, smem, s>>>(a);
  }
  *err = cudaGetLastError();
  return *err == cudaSuccess ? 0 : -1;
}

}  // namespace ftb
