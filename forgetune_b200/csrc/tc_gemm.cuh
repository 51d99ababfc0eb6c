// Tensor-core (tcgen05 / TMEM) GEMM with fp32 accuracy by the 3xTF32 split.
//
//   y[m, n] = epi( sum_k A[m, k] W[k, n] ),   A fp32 [M, K] row-major
//
// Every fp32 value v is split as hi = tf32_round(v) and lo = v - hi (exact),
// and the product is accumulated in fp32 as hi_a*hi_w + hi_a*lo_w + lo_a*hi_w
// (the lo*lo term is below fp32 resolution).  W is split once on the host and
// stored transposed, K-major, as two [N, Kp] arrays; A is split on the fly.
//
// One CTA computes a 128 x BN tile with six warps:
//   warp 0      TMA producer: A tile (fp32) and W_hi / W_lo tiles per k-block
//               of 32, 128-byte swizzled, into a STAGES-deep ring;
//   warp 1      allocates the TMEM accumulator; one thread issues
//               tcgen05.mma (kind::tf32, M=128, N=BN, K=8) three times per
//               k-step and tcgen05.commit frees each stage;
//   warps 2-5   split each A tile in shared memory (hi in place, lo beside
//               it), then run the epilogue: tcgen05.ld of the accumulator,
//               bias / ReLU / residual, stores.
// Every mbarrier wait is bounded: on timeout the kernel records an error
// code, skips the remaining work, waits (bounded) for MMAs in flight,
// releases its TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "epilogue.cuh"

namespace ftb {

struct TcWeights {
  const float* hi = nullptr;  // W^T [N, Kp], tf32-rounded
  const float* lo = nullptr;  // W^T - hi
  int64_t Kp = 0;
  CUtensorMap map_hi[3];      // one per supported BN (64, 128, 256)
  CUtensorMap map_lo[3];
  bool maps_ready = false;
};

struct TcArgs {
  const float* A;
  const float* w_hi;
  const float* w_lo;
  const float* bias;
  const float* res;
  float* Y;
  int64_t M, N, K, Kp;
  uint32_t epi;
};

struct TcKernelParams {
  const float* bias;
  const float* res;
  float* Y;
  int M, N, K;
  uint32_t epi;
  int vec_store;  // Y 16-byte aligned and N % 4 == 0: float4 stores
  int* err;       // device error word: 0 ok, nonzero = a bounded wait gave up
};

constexpr int kTcBK = 32;  // k per stage: one 128-byte swizzle row of fp32
constexpr int kTcBM = 128;

inline int64_t tc_padded_k(int64_t K) { return (K + kTcBK - 1) / kTcBK * kTcBK; }

// shapes the TMA path can address: row stride of A a multiple of 16 bytes
inline bool tc_gemm_supported(int64_t K, int64_t N) { return K % 4 == 0 && K >= kTcBK && N >= 32; }

inline bool tc_gemm_profitable(int64_t M, int64_t K, int64_t N) {
  return M >= 1024 && N >= 64 && K >= 64;
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
// error word) if the phase did not complete within the limit, or if another
// role of this CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kTcWaitLimitNs) {
        *abort_flag = 1;
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// K-major operand tile in the 128-byte swizzle layout TMA wrote: rows of 128 B,
// 8-row groups 1024 B apart.  Start address, leading byte offset 16 B
// (unused by this layout), stride byte offset 1024 B, descriptor version 1,
// layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
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

__device__ __forceinline__ uint32_t tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
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

template <int BN, int STAGES>
struct TcSmem {
  static constexpr int A_BYTES = kTcBM * kTcBK * 4;  // 16 KB
  static constexpr int B_BYTES = BN * kTcBK * 4;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TX_BYTES = A_BYTES + 2 * B_BYTES;  // what TMA writes per stage
  static constexpr int BAR_BYTES = 8 * (3 * STAGES + 2) + 16;
  static constexpr int TOTAL = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_bhi,
               const __grid_constant__ CUtensorMap map_blo, TcKernelParams p) {
  using L = TcSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto a_tile = [&](int s) { return reinterpret_cast<float*>(smem + s * L::STAGE_BYTES); };
  auto alo_tile = [&](int s) { return reinterpret_cast<float*>(smem + s * L::STAGE_BYTES + L::A_BYTES); };
  auto bhi_tile = [&](int s) { return smem + s * L::STAGE_BYTES + 2 * L::A_BYTES; };
  auto blo_tile = [&](int s) { return smem + s * L::STAGE_BYTES + 2 * L::A_BYTES + L::B_BYTES; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * L::STAGE_BYTES);
  uint64_t* full = bars;                 // TMA landed
  uint64_t* conv = bars + STAGES;        // A split into hi / lo
  uint64_t* empty = bars + 2 * STAGES;   // MMAs done reading the stage
  uint64_t* accf = bars + 3 * STAGES;    // accumulator complete
  uint64_t* drain = bars + 3 * STAGES + 1;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 3 * STAGES + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * STAGES + 2) + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTcBM;
  const int n0 = blockIdx.y * BN;
  const int nk = (p.K + kTcBK - 1) / kTcBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    // BN fp32 columns of TMEM for the 128 x BN accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(const_cast<uint32_t*>(tmem_slot))),
                 "r"((uint32_t)BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        const uint32_t r = (uint32_t)(kb / STAGES);
        if (!mbar_wait(&empty[s], (r & 1u) ^ 1u, abort_flag, p.err, 1)) break;
        mbar_arrive_expect_tx(&full[s], L::TX_BYTES);
        tma_load_2d(a_tile(s), &map_a, kb * kTcBK, m0, &full[s]);
        tma_load_2d(bhi_tile(s), &map_bhi, kb * kTcBK, n0, &full[s]);
        tma_load_2d(blo_tile(s), &map_blo, kb * kTcBK, n0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32<BN>();
      bool ok = true;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % STAGES;
        const uint32_t par = (uint32_t)(kb / STAGES) & 1u;
        ok = mbar_wait(&full[s], par, abort_flag, p.err, 2) && mbar_wait(&conv[s], par, abort_flag, p.err, 3);
        if (!ok) break;
        tc_fence_after();
        const uint32_t ahi = smem_u32(a_tile(s)), alo = smem_u32(alo_tile(s));
        const uint32_t bhi = smem_u32(bhi_tile(s)), blo = smem_u32(blo_tile(s));
#pragma unroll
        for (int j = 0; j < kTcBK / 8; ++j) {  // K = 8 tf32 (32 bytes) per MMA
          const uint32_t off = (uint32_t)j * 32u;
          const uint64_t dah = smem_desc_sw128(ahi + off), dal = smem_desc_sw128(alo + off);
          const uint64_t dbh = smem_desc_sw128(bhi + off), dbl = smem_desc_sw128(blo + off);
          umma_tf32(tmem, dah, dbh, idesc, (kb > 0 || j > 0) ? 1u : 0u);
          umma_tf32(tmem, dah, dbl, idesc, 1u);
          umma_tf32(tmem, dal, dbh, idesc, 1u);
        }
        umma_commit(&empty[s]);
      }
      // accumulator ready (or, after an abort, every issued MMA retired)
      umma_commit(ok ? accf : drain);
      if (!ok) mbar_wait(drain, 0, abort_flag, p.err, 4);
    }
  } else {
    // warps 2..5: split A, then the epilogue
    const int t = threadIdx.x - 64;  // 0..127
    bool ok = true;
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % STAGES;
      const uint32_t par = (uint32_t)(kb / STAGES) & 1u;
      ok = mbar_wait(&full[s], par, abort_flag, p.err, 5);
      if (!ok) break;
      float4* hi = reinterpret_cast<float4*>(a_tile(s));
      float4* lo = reinterpret_cast<float4*>(alo_tile(s));
#pragma unroll
      for (int i = 0; i < (kTcBM * kTcBK / 4) / 128; ++i) {
        const int idx = t + i * 128;
        const float4 v = hi[idx];
        float4 h, l;
        h.x = __uint_as_float(tf32_rna(v.x));
        h.y = __uint_as_float(tf32_rna(v.y));
        h.z = __uint_as_float(tf32_rna(v.z));
        h.w = __uint_as_float(tf32_rna(v.w));
        l.x = v.x - h.x;
        l.y = v.y - h.y;
        l.z = v.z - h.z;
        l.w = v.w - h.w;
        hi[idx] = h;
        lo[idx] = l;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
    const bool have_acc = ok && mbar_wait(accf, 0, abort_flag, p.err, 6);
    tc_fence_after();
    __syncwarp();
    if (have_acc) {
      const int q = warp & 3;  // TMEM lane quarter this warp may access
      const int row = q * 32 + lane;
      const int m = m0 + row;
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        __syncwarp();  // tcgen05.ld is warp-collective
        FTB_TMEM_LD32(base + (uint32_t)c, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (m < p.M) {
          const int nb = n0 + c;
          float* yrow = p.Y + (int64_t)m * p.N;
          if (nb + 32 <= p.N && p.vec_store) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              float4 o;
              o.x = apply_epilogue(__uint_as_float(r[j + 0]), p.epi, p.bias, p.res, m, nb + j + 0, p.N);
              o.y = apply_epilogue(__uint_as_float(r[j + 1]), p.epi, p.bias, p.res, m, nb + j + 1, p.N);
              o.z = apply_epilogue(__uint_as_float(r[j + 2]), p.epi, p.bias, p.res, m, nb + j + 2, p.N);
              o.w = apply_epilogue(__uint_as_float(r[j + 3]), p.epi, p.bias, p.res, m, nb + j + 3, p.N);
              *reinterpret_cast<float4*>(yrow + nb + j) = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < p.N)
                yrow[nb + j] = apply_epilogue(__uint_as_float(r[j]), p.epi, p.bias, p.res, m, nb + j, p.N);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN) : "memory");
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
// `ld` floats, box = [box_rows, 32] columns, 128-byte swizzle, zero fill.
inline bool make_map_2d(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  PFN_encodeTiled enc = tma_encoder();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 4) % 16) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline int tc_bn_index(int bn) { return bn == 64 ? 0 : bn == 128 ? 1 : 2; }

// Weight maps for every tile width (built once per replica).
inline bool tc_prepare_weights(TcWeights& w, int64_t N) {
  const int bns[3] = {64, 128, 256};
  for (int i = 0; i < 3; ++i) {
    if (!make_map_2d(&w.map_hi[i], w.hi, N, w.Kp, w.Kp, bns[i])) return false;
    if (!make_map_2d(&w.map_lo[i], w.lo, N, w.Kp, w.Kp, bns[i])) return false;
  }
  w.maps_ready = true;
  return true;
}

// Returns 0 when launched, 1 when this GEMM cannot take the tensor-core path
// (unaligned operand: the caller runs the SIMT kernel), -1 on a launch error.
template <int BN, int STAGES>
inline int launch_tc_bn(const TcArgs& t, const TcWeights& w, int* err, cudaStream_t s) {
  using L = TcSmem<BN, STAGES>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(tc_gemm_kernel<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL) !=
        cudaSuccess)
      return -1;
    attr_set = true;
  }
  CUtensorMap map_a;
  if (!make_map_2d(&map_a, t.A, t.M, t.K, t.K, kTcBM)) return 1;
  TcKernelParams p;
  p.bias = t.bias;
  p.res = t.res;
  p.Y = t.Y;
  p.M = (int)t.M;
  p.N = (int)t.N;
  p.K = (int)t.K;
  p.epi = t.epi;
  p.vec_store = ((reinterpret_cast<uintptr_t>(t.Y) & 15) == 0 && (t.N & 3) == 0) ? 1 : 0;
  p.err = err;
  // the accumulator starts at zero: a bias-first epilogue adds the bias at the end
  if (p.epi & EPI_BIAS_FIRST) p.epi = (p.epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
  dim3 grid((unsigned)((t.M + kTcBM - 1) / kTcBM), (unsigned)((t.N + BN - 1) / BN));
  const int bi = tc_bn_index(BN);
  tc_gemm_kernel<BN, STAGES><<<grid, 192, L::TOTAL, s>>>(map_a, w.map_hi[bi], w.map_lo[bi], p);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

inline int tc_choose_bn(int64_t M, int64_t N, int sm_count) {
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  // wide layers: 256-wide tiles when they still give two full waves
  const int64_t tiles256 = ((M + kTcBM - 1) / kTcBM) * ((N + 255) / 256);
  return tiles256 >= 2 * sm_count ? 256 : 128;
}

inline int launch_tc_gemm(const TcArgs& t, const TcWeights& w, int* err, int sm_count, cudaStream_t s) {
  if (!w.maps_ready || t.M <= 0) return 1;
  if (t.M > 0x7fffffff / 2 || t.N > 65535 * 64) return 1;
  switch (tc_choose_bn(t.M, t.N, sm_count)) {
    case 64: return launch_tc_bn<64, 4>(t, w, err, s);
    case 128: return launch_tc_bn<128, 3>(t, w, err, s);
    default: return launch_tc_bn<256, 2>(t, w, err, s);
  }
}

}  // namespace ftb
