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
// On B200 a dependent L2 round trip costs about 0.6 us (a probe with
// %globaltimer stamps per phase), so the kernel keeps them off each layer's
// critical path: at the start every warp copies the weight rows it will read
// in every layer into shared memory (cp.async, one group per layer; when
// they do not fit, it prefetches them into L2, and into L1 before each
// barrier), and a column's bias and residual are loaded together with its
// weights.  Per layer, a warp owns an output column n at a time and reads
// W's column as the contiguous row n of an fp32 [N, K] copy of the weights
// (float4 loads, eight per lane in flight); the CTA stages the layer's
// input rows [M, K] in shared memory once (L2 loads: the rows were written
// by other SMs in this launch).  Each lane accumulates its k = 4 lane + 128 i
// terms for all M rows; the 32 lane sums of a value are added by a butterfly
// of shuffles, which gives every lane the same bits (fp32 addition is
// commutative), so the result is deterministic run to run.  The association
// of the k terms differs from the per-layer kernels: results agree within
// the tolerance, not bit for bit.
//
// Tagged hand-over (up to 8 rows, when the context has a tag area; at 16
// rows the barrier form measured faster, 20.5 vs 22.3 us for the tiny MLP):
// a layer whose output a
// later layer reads also stores each value as one 64-bit word, the value's
// bits with the launch's tag above them; a reader polls its words (bounded)
// until they carry this launch's tag.  A word is written and read whole, so
// it needs no fence and no barrier: a CTA starts the next layer as soon as
// the values it reads have arrived.  The tag is 0x80000000 | (epoch & 0x7fffffff)
// for a per-context launch counter that the last CTA out advances, so words
// of earlier launches (or of a launch that gave up) never match.
//
// The grid barrier (without a tag area) is a 64-bit arrival counter in the
// context's workspace:
// barrier b of a launch completes when the counter reaches (b + 1) x grid.
// Every CTA increments a second counter as it leaves; the last one resets
// both to zero, so each launch starts from zero, also after a wait that gave
// up.  Waits are bounded (2 s of %globaltimer): a CTA that gives up records
// an error code in the replica's error word and leaves.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "epilogue.cuh"

namespace ftb {

constexpr int kChainMaxLayers = 24;
constexpr int kChainMaxRows = 16;
constexpr int kChainTagRows = 8;  // the tagged hand-over up to this many rows, grid barriers above
constexpr int kChainWarps = 8;
constexpr int kChainSmemBytes = 220 * 1024;  // input rows (M x K floats) and cached weight rows
constexpr unsigned long long kChainWaitNs = 2000000000ull;

struct ChainLayer {
  const float* a;     // [M, K] input rows
  const float* w;     // [N, K] fp32: row n holds column n of W
  const float* bias;  // [N] (or [M, N] with EPI_BIAS_ROWS), or null
  const float* res;   // [M, N] residual, or null
  float* y;           // [M, N]
  int K, N;
  uint32_t epi;       // EPI_* flags; a bias is added after the k sum
  int tag_off;        // this layer's tagged output in ChainParams::tags (words), or -1 (not read by a later layer)
  int a_src;          // the layer whose output `a` is (tagged reads), or -1
  int res_src;        // the layer whose output `res` is (tagged reads), or -1
};

struct ChainParams {
  int n_layers;
  int M;
  unsigned long long* bar;  // [0] arrivals, [1] departures (zero between launches), [3] launch counter
  unsigned long long* tags; // tag area (tagged hand-over), or null (grid barriers)
  unsigned* done;           // mapped host word the last CTA out sets to 1 (output visible), or null
  int* err;                 // the replica's error word (mapped host memory)
  int stall_test;           // failure-detection hook: CTA 0 never arrives at the first barrier
  int xs_floats;            // shared memory for the input rows (floats, a multiple of 4)
  int wcache_per_warp;      // floats of cached weight rows per warp after them (0 = rows stream from L2)
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

__device__ __forceinline__ unsigned long long chain_ld_word(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void chain_st_word(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// The value of a tagged word once it carries `tag` (polled, bounded); false
// when the wait gave up (error code 20 + b recorded) or `*abort` was raised.
__device__ __forceinline__ bool chain_wait_word(const unsigned long long* p, unsigned long long& w, uint32_t tag,
                                                int* err, int b, volatile int* abort) {
  if ((uint32_t)(w >> 32) == tag) return true;
  const unsigned long long t0 = chain_now();
  for (uint32_t it = 0;; ++it) {
    w = chain_ld_word(p);
    if ((uint32_t)(w >> 32) == tag) return true;
    if ((it & 15u) == 15u) {
      if (*abort) return false;
      if (chain_now() - t0 > kChainWaitNs) {
        atomicCAS(err, 0, 20 + b);
        *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void chain_cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
// cp.async.wait_group takes an immediate: wait until at most `pending` of
// this thread's newest groups are still in flight (more than 7: wait for 7)
__device__ __forceinline__ void chain_cp_wait(int pending) {
  switch (pending) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
  }
}

// MB: rows compiled for (M <= MB): the unrolled row loops and the code a
// warp fetches and issues scale with the batch, not with the largest one.
template <int MB>
__global__ void __launch_bounds__(kChainWarps * 32, 1) chain_gemv_kernel(const __grid_constant__ ChainParams p) {
  extern __shared__ float4 chain_smem[];
  float4* chain_xs = chain_smem;  // [M][K/4] of the current layer
  __shared__ int ok_smem;
  __shared__ int abort_smem;  // a tagged wait of this CTA gave up
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kChainWarps + warp;
  const int nw = gridDim.x * kChainWarps;
  const int M = p.M, NL = p.n_layers;
  const bool cached = p.wcache_per_warp > 0;
  float* wcache = reinterpret_cast<float*>(chain_smem) + p.xs_floats + (size_t)warp * p.wcache_per_warp;
  bool ok = !(p.stall_test && blockIdx.x == 0);  // the hook: CTA 0 leaves without arriving (or writing)
  const bool tagged = p.tags != nullptr;
  // this launch's tag (the counter advances when the previous launch's last CTA left)
  const unsigned long long epoch = tagged ? *reinterpret_cast<volatile unsigned long long*>(p.bar + 3) + 1 : 0;
  const uint32_t tag = 0x80000000u | ((uint32_t)epoch & 0x7fffffffu);
  if (threadIdx.x == 0) abort_smem = 0;
  // This warp's weight rows of every layer: copied into shared memory now
  // (one cp.async group per layer, layer 0's first), or, when they do not
  // fit, prefetched into L2.  They do not depend on the activations, so a
  // layer after a barrier waits only on its input rows.
  {
    int off = 0;
    for (int l = 0; l < NL && ok; ++l) {
      const ChainLayer& L = p.layer[l];
      const int K4 = L.K >> 2;
      for (int n = gw; n < L.N; n += nw) {
        if (cached) {
          const float4* src = reinterpret_cast<const float4*>(L.w) + (size_t)n * K4;
          for (int k4 = lane; k4 < K4; k4 += 32) chain_cp_async16(wcache + off + 4 * k4, src + k4);
          off += L.K;
        } else {
          const char* row = reinterpret_cast<const char*>(L.w) + (size_t)n * L.K * 4;
          for (int b = lane * 128; b < L.K * 4; b += 32 * 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(row + b));
        }
      }
      if (cached) asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }
  int woff = 0;
  for (int l = 0; l < NL && ok; ++l) {
    const ChainLayer& L = p.layer[l];
    const int K4 = L.K >> 2, N = L.N;
    const float4* a4 = reinterpret_cast<const float4*>(L.a);
    {
      // the input rows into shared memory: when they take more than one
      // float4 per thread, each thread's loads (up to four) are issued before
      // any of their stores, so a few rows cost one L2 round trip rather than
      // one per row (2 us less per forward of the tiny MLP at 2..16 rows)
      constexpr int SR = 4;
      const int total = M * K4;
      if (tagged && L.a_src >= 0) {
        // from the producing layer's tagged words, as they arrive: up to
        // four words per thread loaded before the first wait
        const unsigned long long* src = p.tags + p.layer[L.a_src].tag_off;
        float* xs = reinterpret_cast<float*>(chain_xs);
        const int words = M * L.K;
        for (int i0 = threadIdx.x; i0 < words && ok; i0 += SR * blockDim.x) {
          unsigned long long t[SR];
#pragma unroll
          for (int r = 0; r < SR; ++r) {
            const int i = i0 + r * blockDim.x;
            t[r] = i < words ? chain_ld_word(src + i) : 0ull;
          }
#pragma unroll
          for (int r = 0; r < SR; ++r) {
            const int i = i0 + r * blockDim.x;
            if (i < words && ok) {
              ok = chain_wait_word(src + i, t[r], tag, p.err, l - 1, &abort_smem);
              xs[i] = __uint_as_float((uint32_t)t[r]);
            }
          }
        }
      } else if (total <= (int)blockDim.x) {
        if ((int)threadIdx.x < total) chain_xs[threadIdx.x] = __ldcg(a4 + threadIdx.x);
      } else {
        for (int i0 = threadIdx.x; i0 < total; i0 += SR * blockDim.x) {
          float4 t[SR];
#pragma unroll
          for (int r = 0; r < SR; ++r) {
            const int i = i0 + r * blockDim.x;
            if (i < total) t[r] = __ldcg(a4 + i);
          }
#pragma unroll
          for (int r = 0; r < SR; ++r) {
            const int i = i0 + r * blockDim.x;
            if (i < total) chain_xs[i] = t[r];
          }
        }
      }
    }
    if (cached) chain_cp_wait(NL - 1 - l);  // this thread's copies of this layer's rows have landed
    __syncthreads();                         // (and every other thread's, and the input rows)
    if (tagged && abort_smem) break;         // a wait of this CTA gave up: leave
    int j = 0;
    for (int n = gw; n < N; n += nw, ++j) {
      const float4* w4 = cached ? reinterpret_cast<const float4*>(wcache + woff + j * L.K)
                                : reinterpret_cast<const float4*>(L.w) + (size_t)n * K4;
      // the epilogue's operands are loaded with the weights, not after the sums
      const int64_t mrow = lane < M ? lane : 0;
      const float bv = L.bias ? ((L.epi & EPI_BIAS_ROWS) ? __ldg(L.bias + mrow * N + n) : __ldg(L.bias + n)) : 0.0f;
      float rv = 0.0f;
      if (L.epi & EPI_RESIDUAL) {
        if (tagged && L.res_src >= 0) {
          // an earlier layer's output, from its tagged words
          const unsigned long long* rp = p.tags + p.layer[L.res_src].tag_off + mrow * N + n;
          unsigned long long w = chain_ld_word(rp);
          if (lane < M && !chain_wait_word(rp, w, tag, p.err, l - 1, &abort_smem)) w = 0ull;
          rv = __uint_as_float((uint32_t)w);
        } else {
          rv = __ldcg(L.res + mrow * N + n);
        }
      }
      float acc[MB];
#pragma unroll
      for (int m = 0; m < MB; ++m) acc[m] = 0.0f;
      // eight float4 of the row per lane in flight at once (K <= 1024 in one round)
      constexpr int WB = 8;
      for (int kb = 0; kb < K4; kb += 32 * WB) {
        float4 wv[WB];
#pragma unroll
        for (int q = 0; q < WB; ++q) {
          const int k4 = kb + 32 * q + lane;
          wv[q] = k4 < K4 ? (cached ? w4[k4] : __ldg(w4 + k4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q = 0; q < WB; ++q) {
          const int k4 = kb + 32 * q + lane;
          if (k4 < K4) {
#pragma unroll
            for (int m = 0; m < MB; ++m) {
              if (m < M) {
                const float4 xv = chain_xs[m * K4 + k4];
                float s = acc[m];
                s = fmaf(xv.x, wv[q].x, s);
                s = fmaf(xv.y, wv[q].y, s);
                s = fmaf(xv.z, wv[q].z, s);
                s = fmaf(xv.w, wv[q].w, s);
                acc[m] = s;
              }
            }
          }
        }
      }
      float mine = 0.0f;  // lane m keeps row m's sum
#pragma unroll
      for (int m = 0; m < MB; ++m) {
        if (m < M) {
          float v = acc[m];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
          if (lane == m) mine = v;
        }
      }
      if (lane < M) {
        float v = mine;
        if (L.bias) v = __fadd_rn(v, bv);
        if (L.epi & EPI_RELU_PRE) v = relu_keep_nan(v);
        if (L.epi & EPI_RESIDUAL) v = __fadd_rn(v, rv);
        if (L.epi & EPI_RELU_POST) v = relu_keep_nan(v);
        L.y[mrow * N + n] = v;
        if (tagged && L.tag_off >= 0)
          chain_st_word(p.tags + L.tag_off + mrow * N + n, ((unsigned long long)tag << 32) | __float_as_uint(v));
      }
    }
    woff += j * L.K;
    if (l + 1 < NL && tagged) {
      __syncthreads();  // every warp is done with this layer's input rows before the next ones land
    } else if (l + 1 < NL) {
      if (!cached) {
        // the next layer's weight rows of this warp into L1 while the barrier waits
        const ChainLayer& Ln = p.layer[l + 1];
        const size_t row_bytes = (size_t)Ln.K * 4;
        for (int n = gw; n < Ln.N; n += nw) {
          const char* row = reinterpret_cast<const char*>(Ln.w) + (size_t)n * row_bytes;
          for (size_t b = (size_t)lane * 128; b < row_bytes; b += 32 * 128)
            asm volatile("prefetch.global.L1 [%0];" ::"l"(row + b));
        }
      }
      ok = chain_grid_sync(p.bar, p.err, l, &ok_smem);
    }
  }
  if (cached) asm volatile("cp.async.wait_group 0;" ::: "memory");  // nothing in flight into shared memory
  // departure: the last CTA out resets both counters for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    // with a completion word, this CTA's output (in mapped host memory) is
    // made visible to the host before it counts itself out
    if (p.done) __threadfence_system();
    else __threadfence();
    const unsigned long long d = atomicAdd(p.bar + 1, 1ull);
    if (d == gridDim.x - 1) {
      atomicExch(p.bar, 0ull);
      atomicExch(p.bar + 1, 0ull);
      if (tagged) atomicExch(p.bar + 3, epoch);  // the next launch tags with epoch + 1
      if (p.done) {
        __threadfence_system();
        *reinterpret_cast<volatile unsigned*>(p.done) = 1u;
      }
    }
  }
}

// Shared memory of a launch over `grid` CTAs: the input rows (M x max K)
// and, when everything fits, each warp's weight rows of every layer.  Fills
// p.xs_floats / p.wcache_per_warp; returns the bytes, or 0 when the input
// rows alone do not fit.
inline size_t chain_plan(ChainParams& p, int grid) {
  int kmax = 0;
  for (int l = 0; l < p.n_layers; ++l) kmax = std::max(kmax, p.layer[l].K);
  p.xs_floats = (p.M * kmax + 3) / 4 * 4;
  const size_t base = (size_t)p.xs_floats * 4;
  if (base > (size_t)kChainSmemBytes) return 0;
  const int nw = grid * kChainWarps;
  int64_t per_warp = 0;
  for (int l = 0; l < p.n_layers; ++l) per_warp += (int64_t)((p.layer[l].N + nw - 1) / nw) * p.layer[l].K;
  per_warp = (per_warp + 3) / 4 * 4;
  const int64_t with_cache = (int64_t)base + (int64_t)kChainWarps * per_warp * 4;
  p.wcache_per_warp = with_cache <= kChainSmemBytes ? (int)per_warp : 0;
  return p.wcache_per_warp ? (size_t)with_cache : base;
}

// Launches the chain on `grid` CTAs (cooperative: all co-resident).
// Returns 0 when launched, -1 on a launch error (kept for take_launch_error).
template <int MB>
inline int launch_chain_mb(const ChainParams& p, int grid, size_t smem, cudaStream_t s) {
  static std::atomic<uint64_t> attr{0};
  cudaError_t e = smem_limit_once(chain_gemv_kernel<MB>, kChainSmemBytes, attr);
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
  return note_launch(cudaLaunchKernelEx(&cfg, chain_gemv_kernel<MB>, p));
}

inline int launch_chain(const ChainParams& p, int grid, size_t smem, cudaStream_t s) {
  if (p.M <= 1) return launch_chain_mb<1>(p, grid, smem, s);
  if (p.M <= 2) return launch_chain_mb<2>(p, grid, smem, s);
  if (p.M <= 4) return launch_chain_mb<4>(p, grid, smem, s);
  if (p.M <= 8) return launch_chain_mb<8>(p, grid, smem, s);
  return launch_chain_mb<16>(p, grid, smem, s);
}

}  // namespace ftb
