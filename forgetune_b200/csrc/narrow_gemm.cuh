// GEMM with few output columns (N <= 16): the small heads of the workloads
// (128 -> 10, 512 -> 10) on many rows.
//
//   y[m, n] = epi( sum_k x[m, k] w[k, n] ),  x [M, K] row-major, w [K, N]
//
// Bound by reading x (4 K bytes per row against 2 K N flops).  A block of
// four warps walks K in chunks of 32: w goes to shared memory (zero-padded to
// NP columns, a multiple of 4), every warp stages its
// 32 rows x 32 k of x through a 32 x 33 tile (each load instruction reads
// 128 contiguous bytes of one row), then each lane -- one row -- accumulates
// its N sums over the chunk's k in order with one FMA per term (k ascending,
// from the bias for a bias-first epilogue, as the SIMT kernel does), reading
// w as broadcast float4s.  Many warps per
// SM hide the shared-memory latency that an epilogue's four warps cannot.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "epilogue.cuh"

namespace ftb {

constexpr int kNarrowMaxN = 16;
constexpr int kNarrowWarps = 4;

// W is staged in K-chunks of kNarrowWChunk rows (the whole W when K fits),
// x in chunks of 32 k: the next x chunk is loaded into registers while the
// current one is used, so one load round trip is exposed per W chunk, not
// per 32 k.
constexpr int kNarrowWChunk = 256;

template <int NP>  // N padded to a multiple of 4
__global__ void __launch_bounds__(kNarrowWarps * 32) narrow_gemm_kernel(const float* __restrict__ x,
                                                                       const float* __restrict__ w,
                                                                       const float* __restrict__ bias,
                                                                       const float* __restrict__ res,
                                                                       float* __restrict__ y, int M, int K, int N,
                                                                       uint32_t epi) {
  __shared__ __align__(16) float ws[kNarrowWChunk * NP];
  __shared__ float xs[kNarrowWarps][32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rows_per_block = kNarrowWarps * 32;
  for (int64_t r0 = (int64_t)blockIdx.x * rows_per_block; r0 < M; r0 += (int64_t)gridDim.x * rows_per_block) {
    const int64_t wr0 = r0 + warp * 32;  // this warp's first row
    const int64_t m = wr0 + lane;        // this lane's row
    float acc[NP];
#pragma unroll
    for (int o = 0; o < NP; ++o) {
      // bias first (the reference's fused loop order): the sums start at it
      acc[o] = 0.0f;
      if ((epi & EPI_BIAS_FIRST) && m < M && o < N) acc[o] = (epi & EPI_BIAS_ROWS) ? bias[m * N + o] : bias[o];
    }
    // x of the first 32-k chunk: row i, column lane
    float xv[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int64_t row = wr0 + i;
      xv[i] = (row < M && lane < K) ? __ldg(x + row * K + lane) : 0.0f;
    }
    for (int kw0 = 0; kw0 < K; kw0 += kNarrowWChunk) {
      const int kwn = min(kNarrowWChunk, K - kw0);
      __syncthreads();  // the previous W chunk is no longer read
      // rows kw0 .. kw0+kwn of w are contiguous: read them flat (coalesced,
      // several loads in flight per thread) into the padded layout
      const float* wsrc = w + (int64_t)kw0 * N;
#pragma unroll 8
      for (int f = threadIdx.x; f < kwn * N; f += blockDim.x) {
        const int kk = f / N, o = f - kk * N;
        ws[kk * NP + o] = __ldg(wsrc + f);
      }
      if (NP != N)
        for (int i = threadIdx.x; i < kwn * (NP - N); i += blockDim.x) {
          const int kk = i / (NP - N), o = N + (i - kk * (NP - N));
          ws[kk * NP + o] = 0.0f;
        }
      __syncthreads();
      for (int k0 = kw0; k0 < kw0 + kwn; k0 += 32) {
        const int kc = min(32, K - k0);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 32; ++i) xs[warp][i][lane] = xv[i];
        __syncwarp();
        // the next chunk's x, in flight while this one is used
        const int kn = k0 + 32;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int64_t row = wr0 + i;
          xv[i] = (row < M && kn + lane < K) ? __ldg(x + row * K + kn + lane) : 0.0f;
        }
        if (m < M) {
          const float4* w4 = reinterpret_cast<const float4*>(ws) + (k0 - kw0) * (NP / 4);
#pragma unroll 8
          for (int kk = 0; kk < kc; ++kk) {
            const float v = xs[warp][lane][kk];
#pragma unroll
            for (int o4 = 0; o4 < NP / 4; ++o4) {
              const float4 c = w4[kk * (NP / 4) + o4];
              acc[4 * o4 + 0] = fmaf(v, c.x, acc[4 * o4 + 0]);
              acc[4 * o4 + 1] = fmaf(v, c.y, acc[4 * o4 + 1]);
              acc[4 * o4 + 2] = fmaf(v, c.z, acc[4 * o4 + 2]);
              acc[4 * o4 + 3] = fmaf(v, c.w, acc[4 * o4 + 3]);
            }
          }
        }
      }
    }
    if (m < M) {
#pragma unroll
      for (int o = 0; o < NP; ++o)
        if (o < N) y[m * N + o] = apply_epilogue(acc[o], epi, bias, res, m, o, N);
    }
  }
}

// The same product for few rows (fewer row blocks of the kernel above than
// SMs): eight warps share 32 rows and split K into eight contiguous ranges,
// so a row's terms are spread over eight lanes instead of one.  W (K x NP,
// at most kNarrowSplitMaxW floats) is staged once per block; each warp stages
// its rows' x through a 32 x 33 tile per 32 k and accumulates its range in k
// order (lane = row); the eight partial sums of a value are then added in
// warp order (the bias-first start value in warp 0's), so the result is
// deterministic, with a different association of the k terms than the
// one-warp-per-row kernel.
constexpr int kNarrowSplitWarps = 8;
constexpr int kNarrowSplitMaxW = 16384;  // 64 KB of staged W
constexpr int kNarrowSplitXFloats = kNarrowSplitWarps * 32 * 33;

// dynamic shared memory: x tiles [8][32][33] (reused for the partial sums,
// [8][32][NP+1]), then W [K][NP]
template <int NP>
__global__ void __launch_bounds__(kNarrowSplitWarps * 32) narrow_gemm_ksplit_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
    const float* __restrict__ res, float* __restrict__ y, int M, int K, int N, uint32_t epi) {
  extern __shared__ __align__(16) float narrow_smem[];
  static_assert(kNarrowSplitWarps * 32 * (NP + 1) <= kNarrowSplitXFloats, "partials fit the x tiles");
  auto xs = reinterpret_cast<float(*)[32][33]>(narrow_smem);
  auto part = reinterpret_cast<float(*)[32][NP + 1]>(narrow_smem);
  float* ws = narrow_smem + kNarrowSplitXFloats;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int f = threadIdx.x; f < K * NP; f += blockDim.x) {
    const int kk = f / NP, o = f - kk * NP;
    ws[f] = o < N ? __ldg(w + (int64_t)kk * N + o) : 0.0f;
  }
  __syncthreads();
  // this warp's k range: contiguous, 32-aligned starts
  const int kc = ((K + kNarrowSplitWarps - 1) / kNarrowSplitWarps + 31) / 32 * 32;
  const int ka = min(K, warp * kc), kb = min(K, ka + kc);
  for (int64_t r0 = (int64_t)blockIdx.x * 32; r0 < M; r0 += (int64_t)gridDim.x * 32) {
    const int64_t m = r0 + lane;
    float acc[NP];
#pragma unroll
    for (int o = 0; o < NP; ++o) {
      acc[o] = 0.0f;
      if (warp == 0 && (epi & EPI_BIAS_FIRST) && m < M && o < N)
        acc[o] = (epi & EPI_BIAS_ROWS) ? bias[m * N + o] : bias[o];
    }
    for (int k0 = ka; k0 < kb; k0 += 32) {
      const int kn = min(32, kb - k0);
      __syncwarp();
#pragma unroll 8
      for (int i = 0; i < 32; ++i) {
        const int64_t row = r0 + i;
        xs[warp][i][lane] = (row < M && lane < kn) ? __ldg(x + row * K + k0 + lane) : 0.0f;
      }
      __syncwarp();
      if (m < M) {
        const float4* w4 = reinterpret_cast<const float4*>(ws) + k0 * (NP / 4);
#pragma unroll 4
        for (int kk = 0; kk < kn; ++kk) {
          const float v = xs[warp][lane][kk];
#pragma unroll
          for (int o4 = 0; o4 < NP / 4; ++o4) {
            const float4 c = w4[kk * (NP / 4) + o4];
            acc[4 * o4 + 0] = fmaf(v, c.x, acc[4 * o4 + 0]);
            acc[4 * o4 + 1] = fmaf(v, c.y, acc[4 * o4 + 1]);
            acc[4 * o4 + 2] = fmaf(v, c.z, acc[4 * o4 + 2]);
            acc[4 * o4 + 3] = fmaf(v, c.w, acc[4 * o4 + 3]);
          }
        }
      }
    }
    __syncthreads();  // every warp is done with its x tile: the partials take their place
#pragma unroll
    for (int o = 0; o < NP; ++o) part[warp][lane][o] = acc[o];
    __syncthreads();
    // 32 rows x N values, summed over the warps in order
    for (int i = threadIdx.x; i < 32 * N; i += blockDim.x) {
      const int rr = i / N, o = i - rr * N;
      const int64_t row = r0 + rr;
      if (row < M) {
        float v = part[0][rr][o];
#pragma unroll
        for (int q = 1; q < kNarrowSplitWarps; ++q) v = __fadd_rn(v, part[q][rr][o]);
        y[row * N + o] = apply_epilogue(v, epi, bias, res, row, o, N);
      }
    }
    __syncthreads();  // the partials are read before the next row block's x tiles overwrite them
  }
}

// Returns 0 when launched, 1 when the shape is not narrow, -1 on a launch error.
inline int launch_narrow_gemm(const float* x, const float* w, const float* bias, const float* res, float* y,
                              int64_t M, int64_t K, int64_t N, uint32_t epi, int sm, cudaStream_t s) {
  if (N < 1 || N > kNarrowMaxN || M < 1 || K < 1 || M > 0x7fffffff || K > 0x7fffffff) return 1;
  const int64_t blocks = (M + kNarrowWarps * 32 - 1) / (kNarrowWarps * 32);
  const int np = (int)((N + 3) / 4 * 4);
  if (blocks < sm && K >= 64 && K * np <= kNarrowSplitMaxW) {
    // too few row blocks to fill the SMs: split K over eight warps per 32 rows
    const int g = (int)((M + 31) / 32);
    const size_t smem = (size_t)(kNarrowSplitXFloats + K * np) * 4;
    constexpr int kMaxSmem = (kNarrowSplitXFloats + kNarrowSplitMaxW) * 4;
    static std::atomic<uint64_t> attr[4];
    auto go = [&](auto kernel, int slot) {
      cudaError_t e = smem_limit_once(kernel, kMaxSmem, attr[slot]);
      if (e != cudaSuccess) return note_launch(e);
      kernel<<<g, kNarrowSplitWarps * 32, smem, s>>>(x, w, bias, res, y, (int)M, (int)K, (int)N, epi);
      return note_launch(cudaGetLastError());
    };
    switch (np) {
      case 4: return go(narrow_gemm_ksplit_kernel<4>, 0);
      case 8: return go(narrow_gemm_ksplit_kernel<8>, 1);
      case 12: return go(narrow_gemm_ksplit_kernel<12>, 2);
      default: return go(narrow_gemm_ksplit_kernel<16>, 3);
    }
  }
  const int grid = (int)std::min<int64_t>(blocks, (int64_t)sm * 16);
  switch (np) {
    case 4: narrow_gemm_kernel<4><<<grid, kNarrowWarps * 32, 0, s>>>(x, w, bias, res, y, (int)M, (int)K, (int)N, epi); break;
    case 8: narrow_gemm_kernel<8><<<grid, kNarrowWarps * 32, 0, s>>>(x, w, bias, res, y, (int)M, (int)K, (int)N, epi); break;
    case 12: narrow_gemm_kernel<12><<<grid, kNarrowWarps * 32, 0, s>>>(x, w, bias, res, y, (int)M, (int)K, (int)N, epi); break;
    default: narrow_gemm_kernel<16><<<grid, kNarrowWarps * 32, 0, s>>>(x, w, bias, res, y, (int)M, (int)K, (int)N, epi); break;
  }
  return note_launch(cudaGetLastError());
}

}  // namespace ftb
