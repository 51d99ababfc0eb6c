// Tensor-core (tcgen05 / TMEM) GEMM with fp32 accuracy by the 3xTF32 split.
//
//   y[m, n] = epi( sum_k A[m, k] W[k, n] ),   A fp32 [M, K] row-major
//
// Every fp32 value v is split as hi = tf32(v) and lo = tf32(v - hi), both
// rounded to nearest, and the product is accumulated in fp32 as
// hi_a*hi_w + hi_a*lo_w + lo_a*hi_w (the lo*lo term is below fp32
// resolution).  W is split once on the host and stored transposed, K-major,
// as two [N, Kp] arrays; A is split on the fly in shared memory.
//
// Persistent kernel: one CTA per SM walks a static round-robin list of
// 128 x BN output tiles (n fastest, so CTAs working on one row block run
// together and share its A tile through L2).  Ten warps:
//   warp 0      TMA producer: A (fp32), W_hi and W_lo tiles per k-block of
//               16 or 32, 64- or 128-byte swizzled, into a STAGES-deep ring
//               that runs continuously across tiles;
//   warp 1      allocates two TMEM accumulators (2 x BN columns); the warp
//               waits, one elected lane issues tcgen05.mma (kind::tf32,
//               M=128, N=BN, K=8) three times per k-step into the accumulator
//               of the current tile and tcgen05.commit frees each stage /
//               publishes each tile;
//   warps 2-5   split each A tile in shared memory (hi in place, lo beside);
//   warps 6-9   epilogue of the previous tile, overlapping the MMAs of the
//               next: tcgen05.ld (lane = row, 32 columns), bias / ReLU /
//               residual in registers, then a 128-byte-swizzled staging tile
//               per warp and a TMA store (or, for output rows that are not
//               16-byte aligned, a shared-memory transpose and row stores;
//               or, with a fused small head, the head's dot products).
// tc_pair_gemm.cuh runs the same roles on SM pairs (256-row tiles).
// Every mbarrier wait is bounded: on timeout the kernel records an error
// code, skips the remaining work, waits (bounded) for MMAs in flight,
// releases its TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <utility>

#include "epilogue.cuh"

namespace ftb {

struct TcWeights {
  const float* hi = nullptr;  // W^T [N, Kp], tf32-rounded
  const float* lo = nullptr;  // tf32(W^T - hi)
  int64_t Kp = 0;
  CUtensorMap map_hi[2][3];   // [k-block 32 / 16][tile width 64 / 128 / 256]
  CUtensorMap map_lo[2][3];
  bool maps_ready = false;
};

// Small-N head computed in the epilogue: y2[m, :] = epi2(y[m, :] W2 + b2),
// with y never stored (W2 is [N, head_n] row-major, head_n <= 16).
// Launch with programmatic stream serialization (see grid_dep_wait).
template <typename... KArgs, typename... Args>
inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

struct TcHead {
  const float* w = nullptr;
  const float* bias = nullptr;
  float* y = nullptr;
  int n = 0;
  uint32_t epi = 0;
};

struct TcArgs {
  float* ws = nullptr;     // split-K partial sums (SM-pair kernel), ws_floats capacity
  size_t ws_floats = 0;
  const float* A;
  const float* w_hi;
  const float* w_lo;
  const float* bias;
  const float* res;
  float* Y;
  int64_t M, N, K, Kp;
  uint32_t epi;
  TcHead head;
  int stall_test;
};

struct TcKernelParams {
  const float* bias;
  const float* res;
  float* Y;
  int M, N, K;
  uint32_t epi;
  TcHead head;
  int* err;  // device error word: 0 ok, nonzero = a bounded wait gave up
  int y_tma;  // the output has a TMA map (rows 16-byte aligned): TMA-store epilogue
  // SM-pair kernel: tiles from split_from on run as `split` column slices
  int split;
  int split_from;
  // SM-pair kernel, split-K: every tile runs as `ksplit` units of `kb_per`
  // k-blocks each; unit s writes its raw sums to slice s of the output map
  // (a [ksplit, M, N] workspace) and a reduction finishes them
  int ksplit;
  int kb_per;
  // test hook: the MMA thread first waits on a barrier nothing completes, so
  // the bounded wait runs out and the abort path runs (failure-detection tests)
  int stall_test;
};

constexpr int kTcMaxHeadN = 16;
constexpr int kTcMaxHeadK = 256;

constexpr int kTcBK = 32;  // k padding unit: one 128-byte swizzle row of fp32
constexpr int kTcBM = 128;
constexpr int kTcThreads = 320;

inline int64_t tc_padded_k(int64_t K) { return (K + kTcBK - 1) / kTcBK * kTcBK; }

// shapes the TMA path can address: row stride of A a multiple of 16 bytes
inline bool tc_gemm_supported(int64_t K, int64_t N) { return K % 4 == 0 && K >= kTcBK && N >= 32; }

// Shape rule of policy `auto` (the autotuner measures instead): on B200 the
// tensor cores beat the SIMT tile kernel from 17 rows on (tuning runs: 2x at
// 256 rows for 784x256 and 512x512 layers, and a tiny-MLP forward of 17..127
// rows in 51 us against 110 us); up to 16 rows the split-K GEMV wins.
inline bool tc_gemm_profitable(int64_t M, int64_t K, int64_t N) {
  return M > 16 && N >= 64 && K >= 64;
}

// round-to-nearest, ties away from zero, to the 10-bit tf32 mantissa (what
// cvt.rna.tf32.f32 does on the device)
inline float tf32_round_host(float v) {
  uint32_t u;
  std::memcpy(&u, &v, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

// ---------------------------------------------------------------------------
// device helpers (inline PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch.  A kernel launched by pdl_launch may be
// scheduled while the previous kernel in the stream is still finishing: it
// sets up its barriers and TMEM, then grid_dep_wait() returns once that
// kernel has completed and its writes are visible; no global memory is read
// or written before it.  grid_dep_trigger() lets the next such kernel be
// scheduled (its CTAs take SMs as this kernel's CTAs exit).  Without the
// launch attribute both are no-ops.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr uint64_t kTcWaitLimitNs = 2000000000ull;  // 2 s per wait: far beyond any legitimate stall

// Bounded wait.  Returns false (and raises the CTA abort flag and the device
// error word) if the phase did not complete within the limit, or, unless
// `ignore_abort`, if another role of this CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code, bool ignore_abort = false) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (!ignore_abort && *abort_flag) return false;
      if (global_ns() - t0 > kTcWaitLimitNs) {
        *abort_flag = 1;
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

// mbar_wait by every lane of a warp, with one outcome for the whole warp.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                               int code, bool ignore_abort = false) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err, code, ignore_abort);
  return __all_sync(0xffffffffu, ok);
}

// One lane of a converged warp (elect.sync): the same lane on every call.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred P;\n\t.reg .b32 R;\n\t"
      "elect.sync R|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// L2 eviction priorities for TMA traffic: streamed operands read once go
// first, weights every tile re-reads and outputs the next layer reads stay.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// K-major operand tile in the swizzle layout TMA wrote: rows of BK*4 bytes
// (128 B for BK=32, 64 B for BK=16), 8-row groups 8*BK*4 bytes apart.  Start
// address, leading byte offset 16 B (unused by these layouts), stride byte
// offset, descriptor version 1, layout type 2 (SWIZZLE_128B) or 4 (SWIZZLE_64B).
template <int BK>
__device__ __forceinline__ uint64_t smem_desc_sw(uint32_t saddr) {
  static_assert(BK == 32 || BK == 16, "k-block of 32 or 16 fp32");
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)((8u * BK * 4u) >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(BK == 32 ? 2 : 4) << 61;
  return d;
}

// Instruction descriptor: D f32, A/B tf32, both K-major, M=128, N=BN.
template <int BN>
__device__ __forceinline__ uint32_t idesc_tf32() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ float tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}

// The low part of a 3xTF32 split, rem = v - tf32_rna(v), rounded the same
// way (to nearest, ties away from zero) with integer operations on its bit
// pattern: half the weight of the 13 dropped mantissa bits is added to the
// magnitude and the bits are cleared, a carry moving into the exponent as
// rounding does.  For every finite rem this gives the bits of cvt.rna.tf32;
// it runs on the integer pipe, so a split costs one conversion per value on
// the quarter-rate conversion pipe instead of two.  rem is finite whenever
// v is; for v = +-Inf (rem NaN) the result is a zero.
__device__ __forceinline__ float tf32_rna_rem(float rem) {
  return __uint_as_float((__float_as_uint(rem) + 0x1000u) & 0xFFFFE000u);
}

#define FTB_TMEM_LD32(taddr, r)                                                                              \
  asm volatile(                                                                                              \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17," \
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                     \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),      \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),          \
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),          \
        "=r"(r[30]), "=r"(r[31])                                                                             \
      : "r"(taddr))

// Split the A values of one stage into tf32 hi (in place) and lo; 128
// threads, N4 float4 each.
template <int N4>
__device__ __forceinline__ void tc_split_a(float4* hi, float4* lo, int t128) {
#pragma unroll
  for (int i = 0; i < N4; ++i) {
    const int idx = t128 + i * 128;
    const float4 v = hi[idx];
    float4 h, l;
    h.x = tf32_rna(v.x);
    h.y = tf32_rna(v.y);
    h.z = tf32_rna(v.z);
    h.w = tf32_rna(v.w);
    l.x = tf32_rna_rem(v.x - h.x);
    l.y = tf32_rna_rem(v.y - h.y);
    l.z = tf32_rna_rem(v.z - h.z);
    l.w = tf32_rna_rem(v.w - h.w);
    hi[idx] = h;
    lo[idx] = l;
  }
}

// Shared-memory views of one epilogue warp.
struct TcEpiSmem {
  float* tr;             // this warp's 32 x 33 transpose tile
  float* stage;          // this warp's 32 x 32 TMA-store tile (1024-byte aligned; overlaps the transpose tiles)
  const float* head_w;   // head weights [N][hp], zero padded
  const float* bias_a;   // bias of this GEMM as the head path reads it
  const float* head_bb;  // bias of the head, [hp]
  int hn, hp;            // head width, padded to whole float4s
};

// Run by the four epilogue warps (threads 192..319): stage the head weights
// and both biases once (all four warps read them).
// `epi` is the 1024-byte aligned epilogue area (4 x 32 x 33 floats) and
// `w` this warp's index among the four.
__device__ __forceinline__ TcEpiSmem tc_epi_setup(const TcKernelParams& p, float* epi, int w, float* head_smem) {
  TcEpiSmem e;
  e.tr = epi + w * 32 * 33;
  e.stage = epi + w * 32 * 32;
  e.hn = p.head.n;
  e.hp = (e.hn + 3) & ~3;
  float* head_w = head_smem;
  float* head_ba = head_smem + kTcMaxHeadK * kTcMaxHeadN;  // bias of this GEMM, [N]
  float* head_bb = head_ba + kTcMaxHeadK;                  // bias of the head, [hp]
  e.head_w = head_w;
  e.head_bb = head_bb;
  e.bias_a = head_ba;  // a column bias; an [M, N] bias is read from global memory
  if (e.hn > 0) {
    const int hn = e.hn, hp = e.hp;
    for (int i = threadIdx.x - 192; i < p.N * hp; i += 128) {
      const int k = i / hp, o = i - k * hp;
      head_w[i] = o < hn ? p.head.w[k * hn + o] : 0.0f;
    }
    for (int i = threadIdx.x - 192; i < p.N; i += 128)
      head_ba[i] = (p.bias && !(p.epi & EPI_BIAS_ROWS)) ? p.bias[i] : 0.0f;
    for (int i = threadIdx.x - 192; i < hp; i += 128) head_bb[i] = (p.head.bias && i < hn) ? p.head.bias[i] : 0.0f;
    asm volatile("bar.sync 1, 128;" ::: "memory");
  }
  return e;
}

// src[4 i .. 4 i + 3] of a run of 32 floats: one four-wide load when `vec`
// (all 32 in bounds and src 16-byte aligned), else the elements below cnt
// and zeros.
__device__ __forceinline__ float4 ld4(const float* src, int i, bool vec, int cnt) {
  if (vec) return reinterpret_cast<const float4*>(src)[i];
  float4 t;
  t.x = 4 * i + 0 < cnt ? src[4 * i + 0] : 0.0f;
  t.y = 4 * i + 1 < cnt ? src[4 * i + 1] : 0.0f;
  t.z = 4 * i + 2 < cnt ? src[4 * i + 2] : 0.0f;
  t.w = 4 * i + 3 < cnt ? src[4 * i + 3] : 0.0f;
  return t;
}

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The epilogue of apply_epilogue on columns 4 i .. 4 i + 3 of a run of 32
// consecutive columns of row m held by this lane: per element the same
// operations in the same order, so the bits are the same.  bsrc points at the
// bias of the run's first column (a column bias: the same address in every
// lane, a broadcast; or the [M, N] bias at [m, n]), rsrc at the residual
// [m, n]; bvec / rvec: four-wide loads allowed; cnt = columns in range.
__device__ __forceinline__ void epi_group(float (&e)[4], uint32_t epi, const float* bsrc, bool bvec,
                                          const float* rsrc, bool rvec, int i, int cnt) {
  // flags as predicates: every step is a select, so the unrolled loops stay
  // one basic block and the loads can be scheduled early
  const bool bias = epi & EPI_BIAS_LAST, pre = epi & EPI_RELU_PRE, res = epi & EPI_RESIDUAL,
             post = epi & EPI_RELU_POST;
  const float4 b = bias ? ld4(bsrc, i, bvec, cnt) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 r = res ? ld4(rsrc, i, rvec, cnt) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float bb[4] = {b.x, b.y, b.z, b.w};
  const float rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float v = e[k];
    v = bias ? __fadd_rn(v, bb[k]) : v;
    v = pre ? relu_keep_nan(v) : v;
    v = res ? __fadd_rn(v, rr[k]) : v;
    v = post ? relu_keep_nan(v) : v;
    e[k] = v;
  }
}

// TMA store of a staged box to (column c0, row c1, slice c2) of the output
// map, kept in L2 for its reader (the next layer or the split-K reduction)
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2, %3}], [%4], %5;" ::
                   "l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src)), "l"(l2_evict_last())
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Rows whose N <= BN hidden values stay in TMEM: lane = row m, the head's
// outputs y2[m, o] = epi2(sum_n y[m, n] W2[n, o] + b2[o]) accumulated over n
// in order (the reference's loop order), each y[m, n] finished by the GEMM's
// epilogue four columns at a time and consumed at once.
// ROWS: the bias is [M, N] in global memory, else a column bias staged in
// shared memory (a compile-time choice, so the compiler sees which memory
// each pointer reads and issues shared-memory loads for the staged operands).
template <int HP4, bool FULL, bool ROWS>
__device__ __forceinline__ void head_chunk(float (&acc)[4 * HP4], const uint32_t (&r)[32], const TcKernelParams& p,
                                           const TcEpiSmem& e, int m, int c, int cnt) {
  const uint32_t epi = p.epi;
  const int64_t off = (int64_t)m * p.N + c;
  const float* bsrc = ROWS ? p.bias + off : e.bias_a + c;
  const bool bvec = FULL && aligned16(bsrc);
  const bool rvec = FULL && aligned16(p.res + off);
  const float4* w4 = reinterpret_cast<const float4*>(e.head_w) + (int64_t)c * HP4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v[4] = {__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]), __uint_as_float(r[4 * i + 2]),
                  __uint_as_float(r[4 * i + 3])};
    epi_group(v, epi, bsrc, bvec, p.res + off, rvec, i, FULL ? 32 : cnt);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * i + k;
      if (FULL || j < cnt) {
#pragma unroll
        for (int o4 = 0; o4 < HP4; ++o4) {
          const float4 w = w4[j * HP4 + o4];
          acc[4 * o4 + 0] = fmaf(v[k], w.x, acc[4 * o4 + 0]);
          acc[4 * o4 + 1] = fmaf(v[k], w.y, acc[4 * o4 + 1]);
          acc[4 * o4 + 2] = fmaf(v[k], w.z, acc[4 * o4 + 2]);
          acc[4 * o4 + 3] = fmaf(v[k], w.w, acc[4 * o4 + 3]);
        }
      }
    }
  }
}

// Rows whose N <= BN hidden values stay in TMEM: lane = row m, the head's
// outputs y2[m, o] = epi2(sum_n y[m, n] W2[n, o] + b2[o]) accumulated over n
// in order (the reference's loop order), each y[m, n] finished by the GEMM's
// epilogue four columns at a time and consumed at once.
template <int HP4>
__device__ __forceinline__ void tc_head_rows(const TcKernelParams& p, const TcEpiSmem& e, uint32_t base, int m) {
  float acc[4 * HP4];
#pragma unroll
  for (int o = 0; o < 4 * HP4; ++o) acc[o] = 0.0f;
#pragma unroll 1
  for (int c = 0; c < p.N; c += 32) {
    uint32_t r[32];
    __syncwarp();
    FTB_TMEM_LD32(base + (uint32_t)c, r);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    const int cnt = min(32, p.N - c);
    if (m < p.M) {
      if (p.epi & EPI_BIAS_ROWS)
        head_chunk<HP4, false, true>(acc, r, p, e, m, c, cnt);
      else if (cnt == 32)
        head_chunk<HP4, true, false>(acc, r, p, e, m, c, cnt);
      else
        head_chunk<HP4, false, false>(acc, r, p, e, m, c, cnt);
    }
  }
  if (m < p.M) {
#pragma unroll
    for (int o = 0; o < 4 * HP4; ++o)
      if (o < e.hn) p.head.y[(int64_t)m * e.hn + o] = apply_epilogue(acc[o], p.head.epi, e.head_bb, nullptr, m, o, e.hn);
  }
}

// Epilogue of one 128-row accumulator block: TMEM columns [base, base + BN)
// of this warp's lane quarter q hold rows m0 + 32 q + lane, output columns
// n0 + c.  With a head: y stays in registers and the head's outputs are
// stored.  Otherwise, when the output rows are 16-byte aligned (y_tma), each
// lane finishes its row's 32 columns in registers, writes them into this
// warp's 128-byte-swizzled staging tile and one lane stores the 32 x 32 block
// with TMA (which clips at the matrix edges); else the block is transposed
// through shared memory so each store instruction writes 128 contiguous bytes.
// `epi` replaces p.epi (0 for split-K partial sums, which the reduction
// finishes); `slice` is the split-K slice the TMA store writes.
template <int BN>
__device__ __forceinline__ void tc_epilogue_block(const TcKernelParams& p, const CUtensorMap* map_y,
                                                  const TcEpiSmem& e, uint32_t base, int m0, int n0, int width,
                                                  int q, int lane, uint32_t epi_all, int slice) {
  if (e.hn > 0) {
    const int m = m0 + q * 32 + lane;
    switch (e.hp) {
      case 4: tc_head_rows<1>(p, e, base, m); break;
      case 8: tc_head_rows<2>(p, e, base, m); break;
      case 12: tc_head_rows<3>(p, e, base, m); break;
      default: tc_head_rows<4>(p, e, base, m); break;
    }
    return;
  }
  if (p.y_tma) {
    float* stage = e.stage;  // 32 rows x 128 bytes, 1024-byte aligned
    const int m = m0 + q * 32 + lane;
    const bool row_ok = m < p.M;
#pragma unroll 1
    for (int c = 0; c < width && n0 + c < p.N; c += 32) {
      uint32_t r[32];
      __syncwarp();
      FTB_TMEM_LD32(base + (uint32_t)c, r);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      const int n = n0 + c;
      const int cnt = min(32, p.N - n);
      const int64_t off = (int64_t)(row_ok ? m : 0) * p.N + n;
      // rows past M load nothing of the [M, N] operands; TMA drops them
      const uint32_t epi = row_ok ? epi_all : (epi_all & ~(uint32_t)(EPI_BIAS_ROWS | EPI_RESIDUAL));
      const float* bsrc = (epi & EPI_BIAS_ROWS) ? p.bias + off : p.bias + n;
      const bool bvec = cnt == 32 && aligned16(bsrc);
      const bool rvec = cnt == 32 && aligned16(p.res + off);
      // the previous block's store has finished reading the staging tile
      if (lane == 0) bulk_wait_read();
      __syncwarp();
      float4* row = reinterpret_cast<float4*>(stage + lane * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float v[4] = {__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]), __uint_as_float(r[4 * i + 2]),
                      __uint_as_float(r[4 * i + 3])};
        epi_group(v, epi, bsrc, bvec, p.res + off, rvec, i, cnt);
        row[i ^ (lane & 7)] = make_float4(v[0], v[1], v[2], v[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(map_y, stage, n, m0 + q * 32, slice);
        bulk_commit();
      }
    }
    return;
  }
  float* tr = e.tr;
#pragma unroll 1
  for (int c = 0; c < width; c += 32) {
    uint32_t r[32];
    __syncwarp();  // tcgen05.ld is warp-collective
    FTB_TMEM_LD32(base + (uint32_t)c, r);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    // lane holds row (q*32 + lane), columns c..c+31: transpose through smem
#pragma unroll
    for (int j = 0; j < 32; ++j) tr[lane * 33 + j] = __uint_as_float(r[j]);
    __syncwarp();
    const int n = n0 + c + lane;
    if (n < p.N) {
      const int rows = min(32, p.M - (m0 + q * 32));
      for (int i = 0; i < rows; ++i) {
        const int m = m0 + q * 32 + i;
        p.Y[(int64_t)m * p.N + n] = apply_epilogue(tr[i * 33 + lane], epi_all, p.bias, p.res, m, n, p.N);
      }
    }
  }
}

template <int BN, int BK, int STAGES, int MH>
struct TcSmem {
  static constexpr int A_HALF_BYTES = kTcBM * BK * 4;  // one 128-row half of the A tile
  static constexpr int A_BYTES = MH * A_HALF_BYTES;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TX_BYTES = A_BYTES + 2 * B_BYTES;  // what TMA writes per stage
  static constexpr int EPI_BYTES = 4 * 32 * 33 * 4;       // per epilogue warp: a 32 x 32 transpose tile
  // head weights [256][16], this GEMM's bias [256], the head's bias [16]
  static constexpr int HEAD_BYTES = (kTcMaxHeadK * kTcMaxHeadN + kTcMaxHeadK + kTcMaxHeadN) * 4;
  static constexpr int NBAR = 3 * STAGES + 6;
  static constexpr int BAR_BYTES = 8 * NBAR + 16;
  static constexpr int TOTAL = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + HEAD_BYTES + BAR_BYTES;
};

template <int BN, int BK, int STAGES, int MH>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_bhi,
               const __grid_constant__ CUtensorMap map_blo, const __grid_constant__ CUtensorMap map_y,
               TcKernelParams p) {
  using L = TcSmem<BN, BK, STAGES, MH>;
  static_assert(L::TOTAL <= 227 * 1024, "shared memory budget");
  static_assert(MH == 1 || MH == 2, "tiles of 128 or 256 rows");
  static_assert(2 * MH * BN <= 512, "two accumulators of MH x BN columns must fit in TMEM");
  constexpr int BMT = kTcBM * MH;          // rows per tile
  constexpr uint32_t TMEM_COLS = 2 * MH * BN;
  extern __shared__ uint8_t smem_raw[];
  // aligned by pointer arithmetic on the shared array (not through an
  // integer), so every pointer derived from it stays a shared-memory pointer
  // to the compiler: ld.shared / st.shared rather than generic accesses
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  auto a_tile = [&](int s) { return reinterpret_cast<float*>(smem + s * L::STAGE_BYTES); };
  auto alo_tile = [&](int s) { return reinterpret_cast<float*>(smem + s * L::STAGE_BYTES + L::A_BYTES); };
  auto bhi_tile = [&](int s) { return smem + s * L::STAGE_BYTES + 2 * L::A_BYTES; };
  auto blo_tile = [&](int s) { return smem + s * L::STAGE_BYTES + 2 * L::A_BYTES + L::B_BYTES; };
  float* epi_stage = reinterpret_cast<float*>(smem + STAGES * L::STAGE_BYTES);
  float* head_smem = reinterpret_cast<float*>(smem + STAGES * L::STAGE_BYTES + L::EPI_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * L::STAGE_BYTES + L::EPI_BYTES + L::HEAD_BYTES);
  uint64_t* full = bars;                // TMA landed
  uint64_t* conv = bars + STAGES;       // A split into hi / lo
  uint64_t* empty = bars + 2 * STAGES;  // MMAs done reading the stage
  uint64_t* accf = bars + 3 * STAGES;   // [2] accumulator buffer complete
  uint64_t* acce = accf + 2;            // [2] accumulator buffer drained by the epilogue
  uint64_t* drain = acce + 2;           // MMAs retired after an abort
  uint64_t* never = drain + 1;          // never arrived on (stall_test)
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(never + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(never + 1) + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (p.M + BMT - 1) / BMT;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int ntiles = tiles_m * tiles_n;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    mbar_init(drain, 1);
    mbar_init(never, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(const_cast<uint32_t*>(tmem_slot))),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();
  grid_dep_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // TMA producer: the whole warp runs the loop (so the loop state is
    // warp-uniform); one elected lane issues the copies
    if (lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    // A is read once when one tile spans all of N (evict it first, keeping the
    // weights and the previous layer's output resident); the weights are
    // re-read by every tile
    const uint64_t pol_a = tiles_n == 1 ? l2_evict_first() : l2_evict_normal();
    const uint64_t pol_w = l2_evict_last();
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int m0 = (t / tiles_n) * BMT;
      const int n0 = (t % tiles_n) * BN;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        const uint32_t r = it / STAGES;
        if (!(ok = mbar_wait_warp(&empty[s], (r & 1u) ^ 1u, abort_flag, p.err, 1))) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full[s], L::TX_BYTES);
          tma_load_2d_hint(a_tile(s), &map_a, kb * BK, m0, &full[s], pol_a);
          tma_load_2d_hint(bhi_tile(s), &map_bhi, kb * BK, n0, &full[s], pol_w);
          tma_load_2d_hint(blo_tile(s), &map_blo, kb * BK, n0, &full[s], pol_w);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // MMA issuer: the whole warp waits and computes descriptors; one elected
    // lane issues the MMAs and the commits that track them.  It waits only
    // for the converters: they arrive after waiting for the whole stage
    // (A and both W halves) to land, so their arrival orders the W copies
    // before the MMAs too.
    const uint32_t idesc = idesc_tf32<BN>();
    uint32_t it = 0, tc = 0;
    bool ok = true;
    if (p.stall_test) ok = mbar_wait_warp(never, 0, abort_flag, p.err, 9);
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
      const uint32_t buf = tc & 1u, use = tc >> 1;
      if (!(ok = mbar_wait_warp(&acce[buf], (use & 1u) ^ 1u, abort_flag, p.err, 2))) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * (uint32_t)(MH * BN);
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        const uint32_t par = (it / STAGES) & 1u;
        if (!(ok = mbar_wait_warp(&conv[s], par, abort_flag, p.err, 4))) break;
        tc_fence_after();
        const uint32_t ahi = smem_u32(a_tile(s)), alo = smem_u32(alo_tile(s));
        const uint32_t bhi = smem_u32(bhi_tile(s)), blo = smem_u32(blo_tile(s));
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < BK / 8; ++j) {  // K = 8 tf32 (32 bytes) per MMA
            const uint32_t off = (uint32_t)j * 32u;
            const uint64_t dbh = smem_desc_sw<BK>(bhi + off), dbl = smem_desc_sw<BK>(blo + off);
#pragma unroll
            for (int h = 0; h < MH; ++h) {  // each 128-row half of the tile against the same W k-block
              const uint32_t ao = off + (uint32_t)(h * L::A_HALF_BYTES);
              const uint64_t dah = smem_desc_sw<BK>(ahi + ao), dal = smem_desc_sw<BK>(alo + ao);
              const uint32_t dh = d + (uint32_t)(h * BN);
              umma_tf32(dh, dah, dbh, idesc, (kb > 0 || j > 0) ? 1u : 0u);
              umma_tf32(dh, dah, dbl, idesc, 1u);
              umma_tf32(dh, dal, dbh, idesc, 1u);
            }
          }
          umma_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (ok) {
        if (elect_one()) umma_commit(&accf[buf]);
        __syncwarp();
      }
    }
    if (!ok) {
      // every MMA issued so far retires before this arrives; wait for it
      // even though the CTA is aborting, so TMEM is not freed under them
      if (elect_one()) umma_commit(drain);
      __syncwarp();
      mbar_wait_warp(drain, 0, abort_flag, p.err, 5, /*ignore_abort=*/true);
    }
  } else if (warp < 6) {
    // warps 2..5: split A into tf32 hi (in place) and lo
    const int t128 = threadIdx.x - 64;
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        if (!(ok = mbar_wait_warp(&full[s], (it / STAGES) & 1u, abort_flag, p.err, 6))) break;
        tc_split_a<(BMT * BK / 4) / 128>(reinterpret_cast<float4*>(a_tile(s)), reinterpret_cast<float4*>(alo_tile(s)),
                                         t128);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
    }
  } else {
    // warps 6..9: epilogue, one TMEM lane quarter each
    const int q = warp & 3;
    const TcEpiSmem e = tc_epi_setup(p, epi_stage, warp - 6, head_smem);
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const uint32_t buf = tc & 1u, use = tc >> 1;
      if (!mbar_wait_warp(&accf[buf], use & 1u, abort_flag, p.err, 7)) break;
      tc_fence_after();
      const int n0 = (t % tiles_n) * BN;
#pragma unroll 1
      for (int h = 0; h < MH; ++h) {
        const int m0 = (t / tiles_n) * BMT + h * kTcBM;
        tc_epilogue_block<BN>(p, &map_y, e, tmem + (buf * MH + h) * (uint32_t)BN + ((uint32_t)(q * 32) << 16), m0,
                              n0, BN, q, lane, p.epi, 0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[buf]);
    }
    if (lane == 0) bulk_wait_all();  // this warp's output stores are complete before the CTA leaves
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// Split-K reduction: y[m, n] = epi(sum over s = 0 .. S-1, in order, of
// part[s, m, n]); four columns per thread.
__global__ void __launch_bounds__(256) tc_splitk_reduce_kernel(const float* __restrict__ part, int S, int M, int N,
                                                               uint32_t epi, const float* __restrict__ bias,
                                                               const float* __restrict__ res, float* __restrict__ Y) {
  const int64_t quads = (int64_t)M * (N / 4);
  const int64_t plane = (int64_t)M * N;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < quads; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = q / (N / 4);
    const int n = (int)(q - m * (N / 4)) * 4;
    const int64_t off = m * N + n;
    float4 acc = *reinterpret_cast<const float4*>(part + off);
    for (int s = 1; s < S; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(part + s * plane + off);
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    float4 out;
    out.x = apply_epilogue(acc.x, epi, bias, res, m, n + 0, N);
    out.y = apply_epilogue(acc.y, epi, bias, res, m, n + 1, N);
    out.z = apply_epilogue(acc.z, epi, bias, res, m, n + 2, N);
    out.w = apply_epilogue(acc.w, epi, bias, res, m, n + 3, N);
    *reinterpret_cast<float4*>(Y + off) = out;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline PFN_encodeTiled tma_encoder() {
  static PFN_encodeTiled fn = []() -> PFN_encodeTiled {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_encodeTiled>(f);
  }();
  return fn;
}

// 2-D fp32 tensor map over a row-major [rows, cols] matrix with row stride
// `ld` floats, box = [box_rows, bk] columns, bk*4-byte swizzle, zero fill.
inline bool make_map_2d(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                        int bk) {
  PFN_encodeTiled enc = tma_encoder();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 4) % 16) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)bk, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Output map: [slices, rows, cols] fp32 row-major, box 32 x 32 x 1, 128-byte
// swizzle (the epilogue's staging tile layout).  Rows are clipped per slice.
inline bool make_map_3d_out(CUtensorMap* map, float* base, int64_t slices, int64_t rows, int64_t cols) {
  PFN_encodeTiled enc = tma_encoder();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 4) % 16) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)slices};
  cuuint64_t strides[2] = {(cuuint64_t)(cols * 4), (cuuint64_t)(rows * cols * 4)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline int tc_bk_index(int bk) { return bk == 32 ? 0 : 1; }

inline int tc_bn_index(int bn) { return bn == 64 ? 0 : bn == 128 ? 1 : 2; }

// Weight maps for every tile width (built once per replica).
inline bool tc_prepare_weights(TcWeights& w, int64_t N) {
  const int bns[3] = {64, 128, 256};
  const int bks[2] = {32, 16};
  for (int b = 0; b < 2; ++b)
    for (int i = 0; i < 3; ++i) {
      if (!make_map_2d(&w.map_hi[b][i], w.hi, N, w.Kp, w.Kp, bns[i], bks[b])) return false;
      if (!make_map_2d(&w.map_lo[b][i], w.lo, N, w.Kp, w.Kp, bns[i], bks[b])) return false;
    }
  w.maps_ready = true;
  return true;
}

// Returns 0 when launched, 1 when this GEMM cannot take the tensor-core path
// (unaligned operand: the caller runs the SIMT kernel), -1 on a launch error.
template <int BN, int BK, int STAGES, int MH>
inline int launch_tc_bn(const TcArgs& t, const TcWeights& w, int* err, int sm_count, cudaStream_t s) {
  using L = TcSmem<BN, BK, STAGES, MH>;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  if (!(attr_set.load() & (1ull << dev))) {
    if (cudaFuncSetAttribute(tc_gemm_kernel<BN, BK, STAGES, MH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             L::TOTAL) != cudaSuccess)
      return -1;
    attr_set.fetch_or(1ull << dev);
  }
  CUtensorMap map_a;
  if (!make_map_2d(&map_a, t.A, t.M, t.K, t.K, kTcBM * MH, BK)) return 1;
  TcKernelParams p;
  p.bias = t.bias;
  p.res = t.res;
  p.Y = t.Y;
  p.M = (int)t.M;
  p.N = (int)t.N;
  p.K = (int)t.K;
  p.epi = t.epi;
  p.head = t.head;
  p.err = err;
  p.stall_test = t.stall_test;
  p.split = 1;
  p.split_from = 0;
  // TMA-store epilogue when the output rows are 16-byte aligned (no head:
  // then only the head's small outputs are written)
  CUtensorMap map_y;
  std::memset(&map_y, 0, sizeof(map_y));
  p.y_tma = (t.head.n == 0 && make_map_3d_out(&map_y, t.Y, 1, t.M, t.N)) ? 1 : 0;
  p.ksplit = 1;
  p.kb_per = 0;
  // the accumulator starts at zero: a bias-first epilogue adds the bias at the end
  if (p.epi & EPI_BIAS_FIRST) p.epi = (p.epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
  if (p.head.epi & EPI_BIAS_FIRST) p.head.epi = (p.head.epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
  if (p.head.n > 0 && (t.N > BN || p.head.n > kTcMaxHeadN || t.N > kTcMaxHeadK)) return 1;
  const int64_t ntiles = ((t.M + kTcBM * MH - 1) / (kTcBM * MH)) * ((t.N + BN - 1) / BN);
  const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sm_count);
  const int bi = tc_bn_index(BN);
  const int ki = BK == 32 ? 0 : 1;
  return pdl_launch(tc_gemm_kernel<BN, BK, STAGES, MH>, dim3(grid), dim3(kTcThreads), L::TOTAL, s, map_a,
                    w.map_hi[ki][bi], w.map_lo[ki][bi], map_y, p) == cudaSuccess
             ? 0
             : -1;
}

inline int tc_choose_bn(int64_t M, int64_t N, int sm_count, bool head) {
  (void)M;
  (void)sm_count;
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  // a fused head needs whole rows in one tile; otherwise 256-wide tiles
  // halve the re-reads of A for layers whose width is a multiple of 256
  return (head || N % 256 == 0) ? 256 : 128;
}

}  // namespace ftb
