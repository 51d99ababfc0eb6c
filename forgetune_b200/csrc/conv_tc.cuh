// Convolution on the tensor cores: im2col rows in a workspace, the 3xTF32
// GEMM of tc_gemm.cuh / tc_pair_gemm.cuh, then NCHW.
//
//   col[m, k]  = x[b, ci, oh*sh - ph + kh*dh, ow*sw - pw + kw*dw]   (0 outside)
//                m = (b*Ho + oh)*Wo + ow,  k = (ci*Kh + kh)*Kw + kw  (the
//                reference's loop order, src/codegen.cpp:412-624), k < K;
//                columns K .. Kp-1 are zero
//   out[m, co] = epi( sum_k col[m, k] W[co, k] )    (the GEMM, W = OIHW as [Cout, K])
//   y[b, co, p] = out[b*HoWo + p, co]                (p = oh*Wo + ow)
//
// Both helper kernels move bytes only (HBM-bound); the GEMM is the work.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "simt_gemm.cuh"

namespace ftb {

// A block builds a 32-row x 128-column tile of col (32 consecutive output
// pixels, one chunk of k): warps walk k, lanes the 32 pixels, so each gather
// instruction reads neighbouring pixels of one input plane (coalesced along
// the row of x) and the k-table entry is the same for the warp; the tile goes
// through shared memory (row stride 129 floats: no bank conflicts either way)
// and leaves as 32 row segments of up to 512 contiguous bytes.  32-bit index
// math: a chunk of rows stays below 2^31 elements (checked by the launcher;
// the workspace budget bounds it far lower).
constexpr int kIm2colRows = 32;
constexpr int kIm2colCols = 128;

__global__ void __launch_bounds__(256) im2col_kernel(const float* __restrict__ x, float* __restrict__ col,
                                                     ConvGeom g, int K, int Kp, int rows) {
  __shared__ float tile[kIm2colRows * (kIm2colCols + 1)];
  constexpr int S = kIm2colCols + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int HoWo = g.Ho * g.Wo;
  const int HW = g.H * g.W;
  const int kc = blockIdx.y * kIm2colCols;
  const int kn = min(kIm2colCols, Kp - kc);
  for (int m0 = blockIdx.x * kIm2colRows; m0 < rows; m0 += gridDim.x * kIm2colRows) {
    const int m = m0 + lane;
    const bool live = m < rows;
    const int b = live ? m / HoWo : 0;
    const int p = live ? m - b * HoWo : 0;
    const int oh = p / g.Wo, ow = p - oh * g.Wo;
    const int ih0 = oh * g.sh - g.ph, iw0 = ow * g.sw - g.pw;
    const float* xb = x + (size_t)b * g.Cin * HW + ih0 * g.W + iw0;
#pragma unroll 4
    for (int j = warp; j < kn; j += 8) {
      const int k = kc + j;
      float val = 0.0f;
      if (k < K && live) {
        const int4 t = __ldg(g.ktab + k);  // {ci*H*W + kh*dh*W + kw*dw, kh*dh, kw*dw, 0}
        const int ih = ih0 + t.y, iw = iw0 + t.z;
        if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) val = __ldg(xb + t.x);
      }
      tile[lane * S + j] = val;
    }
    __syncthreads();
    const int n_rows = min(kIm2colRows, rows - m0);
    for (int r = warp; r < n_rows; r += 8) {
      float* out = col + (size_t)(m0 + r) * Kp + kc;
#pragma unroll
      for (int c = lane; c < kIm2colCols; c += 32)
        if (c < kn) out[c] = tile[r * S + c];
    }
    __syncthreads();
  }
}

// [imgs, HoWo, C] -> [imgs, C, HoWo] through 32 x 33 shared-memory tiles:
// coalesced reads along C, coalesced writes along HoWo.
__global__ void __launch_bounds__(256) rows_to_nchw_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                           int HoWo, int C) {
  __shared__ float tile[32][33];
  const int64_t img = blockIdx.z;
  const int p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* s = src + img * (int64_t)HoWo * C;
  float* d = dst + img * (int64_t)HoWo * C;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    const int p = p0 + r, c = c0 + tx;
    if (p < HoWo && c < C) tile[r][tx] = s[(int64_t)p * C + c];
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int c = c0 + r, p = p0 + tx;
    if (p < HoWo && c < C) d[(int64_t)c * HoWo + p] = tile[tx][r];
  }
}

inline int launch_im2col(const float* x, float* col, const ConvGeom& g, int K, int Kp, int64_t rows, int sm,
                         cudaStream_t s) {
  if (rows <= 0 || rows * (int64_t)Kp >= (int64_t)1 << 31) return -1;
  const int chunks = (Kp + kIm2colCols - 1) / kIm2colCols;
  const int64_t tiles = (rows + kIm2colRows - 1) / kIm2colRows;
  const int gx = (int)std::min<int64_t>(tiles, std::max<int64_t>(1, (int64_t)sm * 8 / chunks));
  im2col_kernel<<<dim3(gx, chunks), 256, 0, s>>>(x, col, g, K, Kp, (int)rows);
  return note_launch(cudaGetLastError());
}

inline int launch_rows_to_nchw(const float* src, float* dst, int64_t imgs, int HoWo, int C, cudaStream_t s) {
  if (imgs > 65535) return -1;
  dim3 grid((unsigned)((HoWo + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)imgs);
  rows_to_nchw_kernel<<<grid, 256, 0, s>>>(src, dst, HoWo, C);
  return note_launch(cudaGetLastError());
}

}  // namespace ftb
