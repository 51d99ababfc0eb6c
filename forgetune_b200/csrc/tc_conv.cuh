// Convolution as an implicit GEMM on the tensor cores: no column matrix, no
// layout pass.
//
//   y[b, co, oh, ow] = epi( sum_k col(m, k) W[co, k] ),   m = (b Ho + oh) Wo + ow
//   col(m, k) = x[b, ci, oh sh - ph + kh dh, ow sw - pw + kw dw]   (0 outside the image)
//   k = (ci Kh + kh) Kw + kw   (the reference's loop order, src/codegen.cpp:412-624)
//
// with the 3xTF32 arithmetic of tc_gemm.cuh (W^T = OIHW as [Cout, Kp], split
// into tf32 hi / lo on the host; col split on the fly; fp32 accumulation in
// TMEM).  Persistent, one CTA per SM over 128-pixel x BN-channel tiles, the
// roles of tc_gemm.cuh with the A operand gathered instead of loaded by TMA:
//   warp 0     TMA producer of the W^T k-blocks (16 k, hi and lo, 64-byte
//              swizzle) into a STAGES-deep ring;
//   warp 1     TMEM (two accumulators of BN columns) and the MMAs (one
//              elected lane, tcgen05.mma kind::tf32 M=128 N=BN K=8, three
//              per k-step);
//   warps 2-17 the gather (four warps per scheduler, to hide load latency):
//              thread (r, h) owns pixel m0 + r of the tile and k-chunk h (4 k)
//              of every k-block; it issues its 4 input loads at once (zero
//              padding decided per value from a k-table of {ci H W + kh dh W
//              + kw dw, kh dh, kw dw} staged in shared memory; a value outside
//              the image loads a valid address and is zeroed by a mask),
//              splits them into tf32 hi and lo and writes both 16-byte chunks
//              in the layout TMA's 64-byte swizzle produces (chunk c of row r
//              at chunk position c ^ ((r >> 1) & 3)); the next two k-blocks'
//              values are loaded while this one is written;
//   warps 18-21 epilogue, overlapping the next tile's MMAs: tcgen05.ld (lane =
//              pixel, 32 channels), bias / ReLU / residual in registers, and
//              stores straight to NCHW (for one channel the 32 pixels of a
//              warp are consecutive addresses of one plane).
// Every mbarrier wait is bounded as in tc_gemm.cuh.
#pragma once

#include "tc_gemm.cuh"

namespace ftb {

struct TcConvParams {
  const float* x;    // NCHW input
  const int4* ktab;  // [K] gather table
  const float* bias;  // [Cout] or null
  const float* res;   // NCHW residual (same shape as y) or null
  float* y;           // NCHW output
  int M, N, K;        // pixels B*Ho*Wo, Cout, Cin*Kh*Kw
  int Cin, H, W, Ho, Wo, sh, sw, ph, pw;
  uint32_t epi;       // EPI_* (bias added after the k sum)
  int* err;
  int stall_test;
};

template <int BN, int STAGES>
struct TcConvSmem {
  static constexpr int A_BYTES = kTcBM * 16 * 4;  // one 16-k block of 128 pixels
  static constexpr int B_BYTES = BN * 16 * 4;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TX_BYTES = 2 * B_BYTES;  // what TMA writes per stage
  static constexpr int NBAR = 3 * STAGES + 6;
  static constexpr int BAR_BYTES = 8 * NBAR + 16;
  static constexpr int KTAB_MAX = 1024;  // k-table entries staged in shared memory (K <= 1024)
  static constexpr int KTAB_BYTES = KTAB_MAX * 16;
  static constexpr int TOTAL = 1024 + STAGES * STAGE_BYTES + BAR_BYTES + KTAB_BYTES;
};

constexpr int kConvGatherWarps = 16;                   // 4 per scheduler: latency hiding for the gather
constexpr int kConvThreads = (2 + kConvGatherWarps + 4) * 32;  // producer, MMA, gather, epilogue

// Issues the 4 loads of col(m, k0 .. k0+3) for this thread's pixel at once:
// the k-table comes from shared memory, a value outside the image (or past
// K) loads the image's first element instead and is zeroed later by its bit
// in the returned mask, so no load waits on another.
__device__ __forceinline__ uint32_t conv_gather4(float4& v, const int4* ktab_s, int K, int H, int W, const float* xb,
                                                 int ih0, int iw0, bool live, int k0) {
  uint32_t ok = 0;
  float t[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = k0 + j;
    const int4 e = ktab_s[k < K ? k : 0];
    const int ih = ih0 + e.y, iw = iw0 + e.z;
    const bool in = live && k < K && ih >= 0 && ih < H && iw >= 0 && iw < W;
    const float* a = in ? xb + ((ptrdiff_t)ih0 * W + iw0 + e.x) : xb;
    t[j] = __ldg(a);
    ok |= (in ? 1u : 0u) << j;
  }
  v = make_float4(t[0], t[1], t[2], t[3]);
  return ok;
}

// 16-byte chunk c of row r of a 64-byte-swizzled k-block tile (rows of 64
// bytes): it sits at chunk position c ^ ((r >> 1) & 3).
__device__ __forceinline__ void conv_store_chunk(uint8_t* tile, int r, int c, float4 v) {
  *reinterpret_cast<float4*>(tile + r * 64 + ((c ^ ((r >> 1) & 3)) << 4)) = v;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kConvThreads, 1)
    tc_conv_kernel(const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                   TcConvParams p) {
  using L = TcConvSmem<BN, STAGES>;
  static_assert(L::TOTAL <= 227 * 1024, "shared memory budget");
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  auto a_tile = [&](int s) { return smem + s * L::STAGE_BYTES; };
  auto alo_tile = [&](int s) { return smem + s * L::STAGE_BYTES + L::A_BYTES; };
  auto bhi_tile = [&](int s) { return smem + s * L::STAGE_BYTES + 2 * L::A_BYTES; };
  auto blo_tile = [&](int s) { return smem + s * L::STAGE_BYTES + 2 * L::A_BYTES + L::B_BYTES; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * L::STAGE_BYTES);
  uint64_t* full = bars;                // W k-block landed
  uint64_t* conv = bars + STAGES;       // A gathered and split (one arrival per gather warp)
  uint64_t* empty = bars + 2 * STAGES;  // MMAs done reading the stage
  uint64_t* accf = bars + 3 * STAGES;   // [2] accumulator complete
  uint64_t* acce = accf + 2;            // [2] accumulator drained (4 arrivals)
  uint64_t* drain = acce + 2;           // MMAs retired after an abort
  uint64_t* never = drain + 1;          // never arrived on (stall_test)
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(never + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(never + 1) + 1;
  int4* ktab_s = reinterpret_cast<int4*>(smem + STAGES * L::STAGE_BYTES + L::BAR_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (p.M + kTcBM - 1) / kTcBM;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int ntiles = tiles_m * tiles_n;
  const int nk = (p.K + 15) / 16;
  const int HoWo = p.Ho * p.Wo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], kConvGatherWarps);
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
  // the gather warps stage the k-table (a weight-side constant, K <= KTAB_MAX)
  if (warp >= 2 && warp < 2 + kConvGatherWarps) {
    for (int k = threadIdx.x - 64; k < p.K; k += kConvGatherWarps * 32) ktab_s[k] = __ldg(p.ktab + k);
    asm volatile("bar.sync 2, %0;" ::"n"(kConvGatherWarps * 32) : "memory");
  }

  if (warp == 0) {
    const uint64_t pol_w = l2_evict_last();  // every tile re-reads the weights
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int n0 = (t % tiles_n) * BN;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        if (!(ok = mbar_wait_warp(&empty[s], ((it / STAGES) & 1u) ^ 1u, abort_flag, p.err, 1))) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full[s], L::TX_BYTES);
          tma_load_2d_hint(bhi_tile(s), &map_bhi, kb * 16, n0, &full[s], pol_w);
          tma_load_2d_hint(blo_tile(s), &map_blo, kb * 16, n0, &full[s], pol_w);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    const uint32_t idesc = idesc_tf32<BN>();
    uint32_t it = 0, tc = 0;
    bool ok = true;
    if (p.stall_test) ok = mbar_wait_warp(never, 0, abort_flag, p.err, 9);
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
      const uint32_t buf = tc & 1u, use = tc >> 1;
      if (!(ok = mbar_wait_warp(&acce[buf], (use & 1u) ^ 1u, abort_flag, p.err, 2))) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * (uint32_t)BN;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        if (!(ok = mbar_wait_warp(&conv[s], (it / STAGES) & 1u, abort_flag, p.err, 4))) break;
        tc_fence_after();
        const uint32_t ahi = smem_u32(a_tile(s)), alo = smem_u32(alo_tile(s));
        const uint32_t bhi = smem_u32(bhi_tile(s)), blo = smem_u32(blo_tile(s));
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {  // K = 8 tf32 (32 bytes) per MMA
            const uint32_t off = (uint32_t)j * 32u;
            const uint64_t dbh = smem_desc_sw<16>(bhi + off), dbl = smem_desc_sw<16>(blo + off);
            const uint64_t dah = smem_desc_sw<16>(ahi + off), dal = smem_desc_sw<16>(alo + off);
            umma_tf32(d, dah, dbh, idesc, (kb > 0 || j > 0) ? 1u : 0u);
            umma_tf32(d, dah, dbl, idesc, 1u);
            umma_tf32(d, dal, dbh, idesc, 1u);
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
      if (elect_one()) umma_commit(drain);
      __syncwarp();
      mbar_wait_warp(drain, 0, abort_flag, p.err, 5, /*ignore_abort=*/true);
    }
  } else if (warp < 2 + kConvGatherWarps) {
    // gather warps: thread (r, h) writes k-chunk h (4 k) of pixel row r of
    // every k-block; the next two k-blocks' loads are in flight meanwhile
    // (the pixel's geometry is computed once per tile: the gather is bound
    // by its instruction count, so a per-load index computation costs more
    // than the cross-tile prefetch it would buy)
    const int gt = threadIdx.x - 64;
    const int r = gt & (kTcBM - 1);  // pixel row of the tile
    const int h = gt >> 7;           // 16-byte chunk of the 64-byte k-block row
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int m = (t / tiles_n) * kTcBM + r;
      const bool live = m < p.M;
      const int b = live ? m / HoWo : 0;
      const int pp = live ? m - b * HoWo : 0;
      const int oh = pp / p.Wo, ow = pp - oh * p.Wo;
      const int ih0 = oh * p.sh - p.ph, iw0 = ow * p.sw - p.pw;
      const float* xb = p.x + (size_t)b * p.Cin * p.H * p.W;
      float4 v0, v1, v2;
      uint32_t m0 = conv_gather4(v0, ktab_s, p.K, p.H, p.W, xb, ih0, iw0, live, 4 * h);
      uint32_t m1 = nk > 1 ? conv_gather4(v1, ktab_s, p.K, p.H, p.W, xb, ih0, iw0, live, 16 + 4 * h) : 0u;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        uint32_t m2 = 0;
        if (kb + 2 < nk) m2 = conv_gather4(v2, ktab_s, p.K, p.H, p.W, xb, ih0, iw0, live, (kb + 2) * 16 + 4 * h);
        const float c[4] = {m0 & 1u ? v0.x : 0.0f, m0 & 2u ? v0.y : 0.0f, m0 & 4u ? v0.z : 0.0f,
                            m0 & 8u ? v0.w : 0.0f};
        float hi[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          hi[j] = tf32_rna(c[j]);
          lo[j] = tf32_rna_rem(c[j] - hi[j]);
        }
        const int s = (int)(it % STAGES);
        if (!(ok = mbar_wait_warp(&full[s], (it / STAGES) & 1u, abort_flag, p.err, 6))) break;
        conv_store_chunk(a_tile(s), r, h, make_float4(hi[0], hi[1], hi[2], hi[3]));
        conv_store_chunk(alo_tile(s), r, h, make_float4(lo[0], lo[1], lo[2], lo[3]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
        v0 = v1;
        m0 = m1;
        v1 = v2;
        m1 = m2;
      }
    }
  } else {
    // the last four warps: epilogue, one TMEM lane quarter (32 pixels) each
    const int q = warp & 3;
    const uint32_t lanes = (uint32_t)(q * 32) << 16;
    const bool bias = p.bias != nullptr && (p.epi & EPI_BIAS_LAST);
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const uint32_t buf = tc & 1u, use = tc >> 1;
      if (!mbar_wait_warp(&accf[buf], use & 1u, abort_flag, p.err, 7)) break;
      tc_fence_after();
      const int n0 = (t % tiles_n) * BN;
      const int m = (t / tiles_n) * kTcBM + q * 32 + lane;
      const bool live = m < p.M;
      const int b = live ? m / HoWo : 0;
      const int pp = live ? m - b * HoWo : 0;
      const size_t base = (size_t)b * p.N * HoWo + pp;  // y[b, 0, pp]
#pragma unroll 1
      for (int c = 0; c < BN / 32 && n0 + 32 * c < p.N; ++c) {
        uint32_t rr[32];
        __syncwarp();
        FTB_TMEM_LD32(tmem + buf * (uint32_t)BN + (uint32_t)(32 * c) + lanes, rr);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (live) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int co = n0 + 32 * c + i;
            if (co < p.N) {
              float v = __uint_as_float(rr[i]);
              if (bias) v = __fadd_rn(v, __ldg(p.bias + co));
              if (p.epi & EPI_RELU_PRE) v = relu_keep_nan(v);
              if (p.epi & EPI_RESIDUAL) v = __fadd_rn(v, p.res[base + (size_t)co * HoWo]);
              if (p.epi & EPI_RELU_POST) v = relu_keep_nan(v);
              p.y[base + (size_t)co * HoWo] = v;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

template <int BN, int STAGES>
inline int launch_tc_conv_bn(TcConvParams p, const TcWeights& w, int sm_count, cudaStream_t s) {
  using L = TcConvSmem<BN, STAGES>;
  static std::atomic<uint64_t> attr{0};
  cudaError_t e = smem_limit_once(tc_conv_kernel<BN, STAGES>, L::TOTAL, attr);
  if (e != cudaSuccess) return note_launch(e);
  const int64_t ntiles = ((int64_t)(p.M + kTcBM - 1) / kTcBM) * ((p.N + BN - 1) / BN);
  const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sm_count);
  const int bi = tc_bn_index(BN);
  return note_launch(pdl_launch(tc_conv_kernel<BN, STAGES>, dim3(grid), dim3(kConvThreads), L::TOTAL, s,
                                w.map_hi[1][bi], w.map_lo[1][bi], p));
}

// Returns 0 when launched, 1 when the shape does not fit (no weight maps,
// too many pixels for 32-bit indices), -1 on a launch error.
inline int launch_tc_conv(TcConvParams p, const TcWeights& w, int sm_count, cudaStream_t s) {
  if (!w.maps_ready || p.M <= 0 || p.N <= 0 || p.K <= 0 || p.K > TcConvSmem<64, 8>::KTAB_MAX) return 1;
  // the accumulator starts at zero: a bias-first epilogue adds the bias at the end
  if (p.epi & EPI_BIAS_FIRST) p.epi = (p.epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
  if (p.N <= 64) return launch_tc_conv_bn<64, 8>(p, w, sm_count, s);
  if (p.N <= 128) return launch_tc_conv_bn<128, 6>(p, w, sm_count, s);
  return launch_tc_conv_bn<256, 4>(p, w, sm_count, s);
}

}  // namespace ftb
