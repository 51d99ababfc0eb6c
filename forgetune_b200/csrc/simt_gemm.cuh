// SIMT fp32 GEMM / implicit-GEMM convolution with a fused epilogue.
//
//   y[m, n] = epi( sum_k A[m, k] * B[k, n] )
//
// A is either a dense row-major [M, K] activation or, for convolution, the
// implicit im2col view of an NCHW input (zero outside the padded window, so
// no padding buffer is materialised).  B is W[K, N] row-major, the layout the
// reference keeps Linear weights in (W^T), or the transposed OIHW conv weight.
//
// Every output is accumulated by one thread in k order 0..K-1, so the result
// of a row does not depend on the tile shape, the batch size or the grid: a
// run is bitwise reproducible and a row computed at B=1 equals the same row
// computed inside B=65536.  With EXACT the product and the sum are separately
// rounded (__fmul_rn / __fadd_rn) and the accumulator starts at the bias or
// at zero exactly as the reference's generated loops do, which makes the
// output bit-identical to the reference CPU runtime; without EXACT the inner
// step is one FFMA.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "epilogue.cuh"

namespace ftb {

struct ConvGeom {
  int Cin, H, W, Cout, Kh, Kw, Ho, Wo;
  int sh, sw, ph, pw, dh, dw;
  const int4* ktab;  // per k: {ci*H*W + kh*dh*W + kw*dw, kh*dh, kw*dw, 0}
};

struct GemmArgs {
  const float* A;
  const float* B;  // [K, N]
  const float* bias;
  const float* res;
  float* Y;
  int M, N, K;
  uint32_t epi;
  ConvGeom conv;
};

// thread-owned row / column index inside the tile: 8-wide micro-tiles are
// split into two 4-wide halves half a tile apart, which keeps the float4
// shared-memory reads of a warp conflict-free
template <int T, int TILE>
__device__ __forceinline__ int micro_index(int t, int i) {
  if constexpr (T >= 8) {
    return (i >> 2) * (TILE / 2) + t * 4 + (i & 3);
  } else {
    return t * T + i;
  }
}

template <int BM, int BN, int BK, int TM, int TN, bool EXACT, bool CONV>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
simt_gemm_kernel(GemmArgs p) {
  constexpr int TX = BN / TN;  // threads along N
  constexpr int TY = BM / TM;  // threads along M
  constexpr int NT = TX * TY;
  static_assert(TM <= 4 || TM == 8, "TM must be <= 4 or 8");
  static_assert(TN <= 4 || TN == 8, "TN must be <= 4 or 8");
  // tile elements each thread stages (small tiles leave some threads idle)
  constexpr int A_PER = (BM * BK + NT - 1) / NT;
  constexpr int B_PER = (BK * BN + NT - 1) / NT;

  __shared__ __align__(16) float As[2][BK][BM + 4];  // +4: conflict-free transposed stores
  __shared__ __align__(16) float Bs[2][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid % TX;
  const int ty = tid / TX;
  // M tiles on grid.x (up to 2^31-1 blocks), N tiles on grid.y
  const int m0 = blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int M = p.M, N = p.N, K = p.K;

  float acc[TM][TN];
  // accumulator start: the bias (bias-first) or zero
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + micro_index<TM, BM>(ty, i);
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + micro_index<TN, BN>(tx, j);
      float v = 0.0f;
      if ((p.epi & EPI_BIAS_FIRST) && m < M && n < N)
        v = (p.epi & EPI_BIAS_ROWS) ? p.bias[(int64_t)m * N + n] : p.bias[n];
      acc[i][j] = v;
    }
  }

  // A element (m, k) of this tile
  auto load_a = [&](int m, int k) -> float {
    if (m >= M || k >= K) return 0.0f;
    if constexpr (CONV) {
      const ConvGeom& c = p.conv;
      const int hw = c.Ho * c.Wo;
      const int b = m / hw;
      const int r = m - b * hw;
      const int ho = r / c.Wo;
      const int wo = r - ho * c.Wo;
      const int4 t = c.ktab[k];
      const int hi = ho * c.sh - c.ph + t.y;
      const int wi = wo * c.sw - c.pw + t.z;
      if (hi < 0 || hi >= c.H || wi < 0 || wi >= c.W) return 0.0f;
      return __ldg(p.A + (int64_t)b * c.Cin * c.H * c.W + (int64_t)(ho * c.sh - c.ph) * c.W +
                   (wo * c.sw - c.pw) + t.x);
    } else {
      return __ldg(p.A + (int64_t)m * K + k);
    }
  };

  float ra[A_PER];
  float rb[B_PER];
  // A tile mapping: consecutive threads walk m (coalesced gathers along W for
  // conv; K-contiguous rows are read BK at a time for dense)
  auto fetch = [&](int k0) {
#pragma unroll
    for (int e = 0; e < A_PER; ++e) {
      const int idx = tid + e * NT;
      if (idx >= BM * BK) break;
      int ml, kl;
      if constexpr (CONV) {
        ml = idx % BM;
        kl = idx / BM;
      } else {
        kl = idx % BK;
        ml = idx / BK;
      }
      ra[e] = load_a(m0 + ml, k0 + kl);
    }
#pragma unroll
    for (int e = 0; e < B_PER; ++e) {
      const int idx = tid + e * NT;
      if (idx >= BK * BN) break;
      const int nl = idx % BN;
      const int kl = idx / BN;
      const int k = k0 + kl, n = n0 + nl;
      rb[e] = (k < K && n < N) ? __ldg(p.B + (int64_t)k * N + n) : 0.0f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int e = 0; e < A_PER; ++e) {
      const int idx = tid + e * NT;
      if (idx >= BM * BK) break;
      int ml, kl;
      if constexpr (CONV) {
        ml = idx % BM;
        kl = idx / BM;
      } else {
        kl = idx % BK;
        ml = idx / BK;
      }
      As[buf][kl][ml] = ra[e];
    }
#pragma unroll
    for (int e = 0; e < B_PER; ++e) {
      const int idx = tid + e * NT;
      if (idx >= BK * BN) break;
      Bs[buf][idx / BN][idx % BN] = rb[e];
    }
  };

  const int ktiles = (K + BK - 1) / BK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) fetch((kt + 1) * BK);
    // the last tile may be partial; EXACT must not add products past K
    const int kcount = min(BK, K - kt * BK);
    if (kcount == BK) {
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        float a[TM], b[TN];
#pragma unroll
        for (int i = 0; i < TM; ++i) a[i] = As[buf][kk][micro_index<TM, BM>(ty, i)];
#pragma unroll
        for (int j = 0; j < TN; ++j) b[j] = Bs[buf][kk][micro_index<TN, BN>(tx, j)];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            if constexpr (EXACT)
              acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
            else
              acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
          }
      }
    } else {
      for (int kk = 0; kk < kcount; ++kk) {
        float a[TM], b[TN];
#pragma unroll
        for (int i = 0; i < TM; ++i) a[i] = As[buf][kk][micro_index<TM, BM>(ty, i)];
#pragma unroll
        for (int j = 0; j < TN; ++j) b[j] = Bs[buf][kk][micro_index<TN, BN>(tx, j)];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            if constexpr (EXACT)
              acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
            else
              acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
          }
      }
    }
    if (kt + 1 < ktiles) {
      stash(buf ^ 1);
      __syncthreads();
    }
  }

  // epilogue + store
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + micro_index<TM, BM>(ty, i);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + micro_index<TN, BN>(tx, j);
      if (n >= N) continue;
      float v = apply_epilogue(acc[i][j], p.epi, p.bias, p.res, m, n, N);
      if constexpr (CONV) {
        const int hw = p.conv.Ho * p.conv.Wo;
        const int b = m / hw;
        p.Y[((int64_t)b * N + n) * hw + (m - b * hw)] = v;
      } else {
        p.Y[(int64_t)m * N + n] = v;
      }
    }
  }
}

}  // namespace ftb
