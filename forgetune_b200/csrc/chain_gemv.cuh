// The whole forward pass of a chain of dense layers in one launch, for small
// batches (at most 16 rows): the latency path of the tiny and residual MLPs.
//
//   for each layer l:  y_l[m, n] = epi_l( sum_k a_l[m, k] W_l[k, n] )
//
// where a_l is the network input or an earlier layer's output and the
// epilogue is the engine's (bias, NaN-keeping ReLU, residual, ReLU).  One
// persistent grid (one CTA of eight warps per SM at most, all co-resident:
// a cooperative launch) walks the layers; a layer's outputs are complete
// for every CTA after a grid-wide barrier, so the next layer reads them.
//
// At the start every warp prefetches into L2 the weight rows it will read in
// every layer (they do not depend on the activations), and before each
// barrier the next layer's rows into L1, so after a barrier a layer waits
// only on its input rows.  Per layer, a warp owns an output column n at
// a time and reads W's column as the contiguous row n of an fp32 [N, K] copy
// of the weights (float4 loads, eight per lane in flight); the CTA stages the layer's
// input rows [M, K] in shared memory once (L2 loads: the rows were written
// by other SMs in this launch).  Each lane accumulates its k = 4 lane + 128 i
// terms for all M rows; the 32 lane sums of a value are added by a butterfly
// of shuffles, which gives every lane the same bits (fp32 addition is
// commutative), so the result is deterministic run to run.  The association
// of the k terms differs from the per-layer kernels: results agree within
// the tolerance, not bit for bit.
//
// The grid barrier is a 64-bit arrival counter in the context's workspace:
// barrier b of a launch completes when the counter reaches (b + 1) x grid.
// Every CTA increments a second counter as it leaves; the last one resets
// both to zero, so each launch starts from zero, also after a wait that gave
// up.  Waits are bounded (2 s of %globaltimer): a CTA that gives up records
// an error code in the replica's error word and leaves.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "epilogue.cuh"

namespace ftb {

constexpr int kChainMaxLayers = 24;
constexpr int kChainMaxRows = 16;
constexpr int kChainWarps = 8;
constexpr int kChainSmemBytes = 160 * 1024;  // staged input rows: M x K floats
constexpr unsigned long long kChainWaitNs = 2000000000ull;

struct ChainLayer {
  const float* a;     // [M, K] input rows
  const float* w;     // [N, K] fp32: row n holds column n of W
  const float* bias;  // [N] (or [M, N] with EPI_BIAS_ROWS), or null
  const float* res;   // [M, N] residual, or null
  float* y;           // [M, N]
  int K, N;
  uint32_t epi;       // EPI_* flags; a bias is added after the k sum
  int pad;
};

struct ChainParams {
  int n_layers;
  int M;
  unsigned long long* bar;  // [0] arrivals, [1] departures; zero between launches
  int* err;                 // the replica's error word (mapped host memory)
  int stall_test;           // failure-detection hook: CTA 0 never arrives at the first barrier
  int pad;
  ChainLayer layer[kChainMaxLayers];
};

__device__ __forceinline__ unsigned long long chain_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid-wide barrier number `b` of this launch; false when the wait gave up.
__device__ __forceinline__ bool chain_grid_sync(unsigned long long* bar, int* err, int b, int* ok_smem) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    // the arrival releases this CTA's stores (ordered before it by the CTA barrier)
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
    const unsigned long long target = (unsigned long long)(b + 1) * gridDim.x;
    // poll without sleeping (a sleep's granularity is coarser than the wait)
    const unsigned long long t0 = chain_now();
    for (uint32_t it = 0;; ++it) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(bar) : "memory");
      if (v >= target) break;
      if ((it & 15u) == 15u && chain_now() - t0 > kChainWaitNs) {
        atomicCAS(err, 0, 20 + b);
        ok = 0;
        break;
      }
    }
    __threadfence();
    *ok_smem = ok;
  }
  __syncthreads();
  return *ok_smem != 0;
}

__global__ void __launch_bounds__(kChainWarps * 32, 1) chain_gemv_kernel(const __grid_constant__ ChainParams p) {
  extern __shared__ float4 chain_xs[];  // [M][K/4] of the current layer
  __shared__ int ok_smem;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kChainWarps + warp;
  const int nw = gridDim.x * kChainWarps;
  const int M = p.M;
  bool ok = !(p.stall_test && blockIdx.x == 0);  // the hook: CTA 0 leaves without arriving
  // Every layer's weight rows this warp will read, prefetched into L2 now:
  // they do not depend on the activations, so later layers find them there
  // instead of waiting on HBM after each barrier.
  for (int l = 0; l < p.n_layers && ok; ++l) {
    const ChainLayer& L = p.layer[l];
    const size_t row_bytes = (size_t)L.K * 4;
    for (int n = gw; n < L.N; n += nw) {
      const char* row = reinterpret_cast<const char*>(L.w) + (size_t)n * row_bytes;
      for (size_t b = (size_t)lane * 128; b < row_bytes; b += 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(row + b));
    }
  }
  for (int l = 0; l < p.n_layers && ok; ++l) {
    const ChainLayer& L = p.layer[l];
    const int K4 = L.K >> 2, N = L.N;
    const float4* a4 = reinterpret_cast<const float4*>(L.a);
    for (int i = threadIdx.x; i < M * K4; i += blockDim.x) chain_xs[i] = __ldcg(a4 + i);
    __syncthreads();
    for (int n = gw; n < N; n += nw) {
      const float4* w4 = reinterpret_cast<const float4*>(L.w) + (size_t)n * K4;
      float acc[kChainMaxRows];
#pragma unroll
      for (int m = 0; m < kChainMaxRows; ++m) acc[m] = 0.0f;
      // eight float4 of the row per lane in flight at once (K <= 1024 in one round)
      constexpr int WB = 8;
      for (int kb = 0; kb < K4; kb += 32 * WB) {
        float4 wv[WB];
#pragma unroll
        for (int j = 0; j < WB; ++j) {
          const int k4 = kb + 32 * j + lane;
          wv[j] = k4 < K4 ? __ldg(w4 + k4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < WB; ++j) {
          const int k4 = kb + 32 * j + lane;
          if (k4 < K4) {
#pragma unroll
            for (int m = 0; m < kChainMaxRows; ++m) {
              if (m < M) {
                const float4 xv = chain_xs[m * K4 + k4];
                float s = acc[m];
                s = fmaf(xv.x, wv[j].x, s);
                s = fmaf(xv.y, wv[j].y, s);
                s = fmaf(xv.z, wv[j].z, s);
                s = fmaf(xv.w, wv[j].w, s);
                acc[m] = s;
              }
            }
          }
        }
      }
      float mine = 0.0f;  // lane m keeps row m's sum
#pragma unroll
      for (int m = 0; m < kChainMaxRows; ++m) {
        if (m < M) {
          float v = acc[m];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
          if (lane == m) mine = v;
        }
      }
      if (lane < M) {
        const int64_t m = lane;
        float v = mine;
        if (L.bias) v = __fadd_rn(v, (L.epi & EPI_BIAS_ROWS) ? __ldg(L.bias + m * N + n) : __ldg(L.bias + n));
        if (L.epi & EPI_RELU_PRE) v = relu_keep_nan(v);
        if (L.epi & EPI_RESIDUAL) v = __fadd_rn(v, __ldcg(L.res + m * N + n));
        if (L.epi & EPI_RELU_POST) v = relu_keep_nan(v);
        L.y[m * N + n] = v;
      }
    }
    if (l + 1 < p.n_layers) {
      // the next layer's weight rows of this warp into L1 while the barrier waits
      const ChainLayer& Ln = p.layer[l + 1];
      const size_t row_bytes = (size_t)Ln.K * 4;
      for (int n = gw; n < Ln.N; n += nw) {
        const char* row = reinterpret_cast<const char*>(Ln.w) + (size_t)n * row_bytes;
        for (size_t b = (size_t)lane * 128; b < row_bytes; b += 32 * 128)
          asm volatile("prefetch.global.L1 [%0];" ::"l"(row + b));
      }
      ok = chain_grid_sync(p.bar, p.err, l, &ok_smem);
    }
  }
  // departure: the last CTA out resets both counters for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned long long d = atomicAdd(p.bar + 1, 1ull);
    if (d == gridDim.x - 1) {
      atomicExch(p.bar, 0ull);
      atomicExch(p.bar + 1, 0ull);
    }
  }
}

// Launches the chain on `grid` CTAs (cooperative: all co-resident).
// Returns 0 when launched, -1 on a launch error (kept for take_launch_error).
inline int launch_chain(const ChainParams& p, int grid, size_t smem, cudaStream_t s) {
  static std::atomic<uint64_t> attr{0};
  cudaError_t e = smem_limit_once(chain_gemv_kernel, kChainSmemBytes, attr);
  if (e != cudaSuccess) return note_launch(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kChainWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeCooperative;
  attrs[0].val.cooperative = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  return note_launch(cudaLaunchKernelEx(&cfg, chain_gemv_kernel, p));
}

}  // namespace ftb
