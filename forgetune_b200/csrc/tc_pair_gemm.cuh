// Tensor-core GEMM on SM pairs (tcgen05 cta_group::2): the arithmetic of
// tc_gemm.cuh (3xTF32 split, fp32 accumulation in TMEM, same k order, so the
// results are bit-identical) on 256-row tiles computed by two CTAs.
//
// A cluster of two CTAs computes each 256 x BN output tile with one
// tcgen05.mma.cta_group::2 (M=256, N=BN, K=8) per k-step and split term.
// CTA r holds rows [128 r, 128 r + 128) of the A tile and rows
// [r BN/2, (r+1) BN/2) of the W^T tile at the same shared-memory offsets in
// both CTAs, and its TMEM receives its 128 rows of the accumulator.  Each SM
// therefore loads and serves half of every W k-block that a one-SM 128-row
// tile needs: per MMA it moves two thirds of the operand bytes through shared
// memory, and its stages are smaller, so the ring holds more of them (six
// instead of four at BN=256) and hides more of the load latency.
//
// Roles per CTA (320 threads, as in the one-SM kernel):
//   warp 0     TMA producer for this CTA's A rows and W half, completing on
//              this CTA's own barriers (no multicast);
//   warp 1     TMEM allocation (cta_group::2, both CTAs); in the leader CTA
//              (rank 0) it issues the MMAs of the pair and commits to the
//              stage-free and tile-done barriers of both CTAs;
//   warps 2-5  split this CTA's A rows into tf32 hi / lo, then arrive on the
//              leader's conversion barrier (8 arrivals: 4 warps x 2 CTAs) --
//              they waited for the whole stage to land, so their arrival
//              also orders this CTA's W half before the MMAs;
//   warps 6-9  epilogue of this CTA's 128 rows, then arrive on the leader's
//              accumulator-free barrier (8 arrivals).
// The accumulators take all of TMEM: two buffers of 256 columns or four of
// 128, so at BN=128 a slow epilogue delays the MMAs only three tiles later.
// Waits are bounded as in the one-SM kernel; a CTA that gives up also raises
// its peer's abort flag.  Both CTAs meet at a cluster barrier before TMEM is
// released, so neither leaves while MMAs of the pair may still touch its
// shared memory or TMEM.
#pragma once

#include "tc_gemm.cuh"

namespace ftb {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// shared::cluster address of the shared variable `p` in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Arrive on an mbarrier of this CTA or the peer (default release semantics,
// as for a local arrive: what the arrival publishes to the pair's MMAs is
// shared memory already made visible to the async proxy by
// fence.proxy.async).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

__device__ __forceinline__ void st_cluster_u32(uint32_t caddr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(caddr), "r"(v) : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Bounded wait (arrivals may come from the peer CTA).  On timeout it raises
// this CTA's and the peer's abort flags.
__device__ __forceinline__ bool pair_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint32_t peer_abort,
                                          int* err, int code, bool ignore_abort = false) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (!ignore_abort && *abort_flag) return false;
      if (global_ns() - t0 > kTcWaitLimitNs) {
        *abort_flag = 1;
        st_cluster_u32(peer_abort, 1u);
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool pair_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                               uint32_t peer_abort, int* err, int code, bool ignore_abort = false) {
  const bool ok = pair_wait(bar, parity, abort_flag, peer_abort, err, code, ignore_abort);
  return __all_sync(0xffffffffu, ok);
}

// D[256 x N] (+)= A[256 x 8] B[8 x N] over the SM pair, tf32 operands from
// the shared memory of both CTAs at the same offsets.
__device__ __forceinline__ void umma2_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive once on the mbarrier at shared::cluster address `caddr` (this CTA's
// or the peer's) when every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma2_commit(uint32_t caddr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(caddr)
               : "memory");
}

// Instruction descriptor: D f32, A/B tf32, both K-major, M=256, N=n (a
// multiple of 16, at most 256).
__device__ __forceinline__ uint32_t idesc_tf32_pair(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// The pair's list of work units.  Tiles (256 x BN) run in rounds of
// `npairs`; when the last round is partial, its tiles are cut into `split`
// column slices of BN / split so that more pairs share it (a slice is the
// same MMAs on fewer columns: the results do not change).
// With split-K (ksplit > 1, no column slices) every tile is instead cut
// into ksplit units of kb_per k-blocks, unit s of a tile covering k-blocks
// [s kb_per, (s+1) kb_per) and writing slice s of the partial sums.
struct PairWork {
  int tiles_n;  // tiles per row block
  int full;     // units [0, full) are whole tiles, tile = unit
  int split;    // the tiles from `full` on are cut into this many slices
  int ksplit;   // k ranges per tile (1: none)
  int kb_per;   // k-blocks per range
  int nk;       // k-blocks of the whole K
  int units;
  __device__ __forceinline__ void unit(int u, int bn, int& m0, int& n0, int& width, int& kb0, int& kb1,
                                       int& slice) const {
    int tile = u, part = 0;
    width = bn;
    slice = 0;
    kb0 = 0;
    kb1 = nk;
    if (ksplit > 1) {
      tile = u / ksplit;
      slice = u % ksplit;
      kb0 = slice * kb_per;
      kb1 = min(nk, kb0 + kb_per);
    } else if (u >= full) {
      tile = full + (u - full) / split;
      part = (u - full) % split;
      width = bn / split;
    }
    m0 = (tile / tiles_n) * 256;
    n0 = (tile % tiles_n) * bn + part * width;
  }
};

template <int BN, int BK, int STAGES>
struct TcPairSmem {
  static constexpr int A_BYTES = kTcBM * BK * 4;     // this CTA's 128 rows of the A tile
  static constexpr int B_BYTES = (BN / 2) * BK * 4;  // this CTA's half of the W^T tile
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TX_BYTES = A_BYTES + 2 * B_BYTES;
  static constexpr int EPI_BYTES = 4 * 32 * 33 * 4;
  static constexpr int HEAD_BYTES = (kTcMaxHeadK * kTcMaxHeadN + kTcMaxHeadK + kTcMaxHeadN) * 4;
  static constexpr int NACC = 512 / BN;  // accumulator buffers: all of TMEM (2 of 256 or 4 of 128 columns)
  static constexpr int NBAR = 3 * STAGES + 2 * NACC + 2;
  static constexpr int BAR_BYTES = 8 * NBAR + 16;
  static constexpr int TOTAL = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + HEAD_BYTES + BAR_BYTES;
};

template <int BN, int BK, int STAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    tc_pair_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_bhi,
                        const __grid_constant__ CUtensorMap map_blo, const __grid_constant__ CUtensorMap map_y,
                        TcKernelParams p) {
  using L = TcPairSmem<BN, BK, STAGES>;
  static_assert(L::TOTAL <= 227 * 1024, "shared memory budget");
  static_assert(BN == 128 || BN == 256, "W^T tiles split into two halves of 64 or 128 rows");
  constexpr uint32_t NACC = L::NACC;
  constexpr uint32_t TMEM_COLS = NACC * BN;
  extern __shared__ uint8_t smem_raw[];
  // the same offsets in both CTAs: the pair's MMAs address the peer's tiles
  // through the leader's descriptors
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
  uint64_t* full = bars;                // this CTA's TMA landed
  uint64_t* conv = bars + STAGES;       // leader: A of both CTAs split (8 arrivals)
  uint64_t* empty = bars + 2 * STAGES;  // the pair's MMAs done reading the stage
  uint64_t* accf = bars + 3 * STAGES;   // [NACC] accumulator buffer complete
  uint64_t* acce = accf + NACC;         // [NACC] leader: buffer drained by both epilogues (8 arrivals)
  uint64_t* drain = acce + NACC;        // leader: MMAs retired after an abort
  uint64_t* never = drain + 1;          // never arrived on (stall_test)
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(never + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(never + 1) + 1;

  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (p.M + 255) / 256;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int ntiles = tiles_m * tiles_n;
  const int nk = (p.K + BK - 1) / BK;
  PairWork work;
  work.tiles_n = tiles_n;
  work.nk = nk;
  work.ksplit = p.ksplit > 1 ? p.ksplit : 1;
  work.kb_per = work.ksplit > 1 ? p.kb_per : nk;
  work.split = (p.split > 1 && work.ksplit == 1) ? p.split : 1;
  work.full = work.split > 1 ? p.split_from : ntiles;
  work.units = work.ksplit > 1 ? ntiles * work.ksplit : work.full + (ntiles - work.full) * work.split;
  const int pair = (int)cluster_index();
  const int npairs = (int)cluster_count();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 8);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < (int)NACC; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 8);
    }
    mbar_init(drain, 1);
    mbar_init(never, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(const_cast<uint32_t*>(tmem_slot))),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated before any remote arrival
  tc_fence_after();
  grid_dep_wait();
  grid_dep_trigger();
  const uint32_t tmem = *tmem_slot;
  const uint32_t peer_abort = cluster_addr(const_cast<int*>(abort_flag), peer);

  if (warp == 0) {
    if (lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    // A is read once when one tile spans all of N (evict it first, keeping the
    // weights and the previous layer's output resident); the weights are
    // re-read by every tile
    const uint64_t pol_a = tiles_n == 1 ? l2_evict_first() : l2_evict_normal();
    const uint64_t pol_w = l2_evict_last();
    uint32_t it = 0;
    bool ok = true;
    for (int u = pair; u < work.units && ok; u += npairs) {
      int m0, n0, width, kb0, kb1, slice;
      work.unit(u, BN, m0, n0, width, kb0, kb1, slice);
      m0 += (int)rank * kTcBM;
      // this CTA's half of the unit's W^T rows (a narrower slice loads the
      // full BN/2-row box; the MMA reads only its first width/2 rows)
      const int nb = n0 + (int)rank * (width / 2);
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        const uint32_t r = it / STAGES;
        if (!(ok = pair_wait_warp(&empty[s], (r & 1u) ^ 1u, abort_flag, peer_abort, p.err, 1))) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full[s], L::TX_BYTES);
          tma_load_2d_hint(a_tile(s), &map_a, kb * BK, m0, &full[s], pol_a);
          tma_load_2d_hint(bhi_tile(s), &map_bhi, kb * BK, nb, &full[s], pol_w);
          tma_load_2d_hint(blo_tile(s), &map_blo, kb * BK, nb, &full[s], pol_w);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      uint32_t it = 0, tc = 0;
      bool ok = true;
      if (p.stall_test) ok = pair_wait_warp(never, 0, abort_flag, peer_abort, p.err, 9);
      for (int u = pair; u < work.units && ok; u += npairs, ++tc) {
        int m0, n0, width, kb0, kb1, slice;
        work.unit(u, BN, m0, n0, width, kb0, kb1, slice);
        const uint32_t idesc = idesc_tf32_pair(width);
        const uint32_t buf = tc % NACC, use = tc / NACC;
        if (!(ok = pair_wait_warp(&acce[buf], (use & 1u) ^ 1u, abort_flag, peer_abort, p.err, 2))) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * (uint32_t)BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = (int)(it % STAGES);
          const uint32_t par = (it / STAGES) & 1u;
          if (!(ok = pair_wait_warp(&conv[s], par, abort_flag, peer_abort, p.err, 4))) break;
          tc_fence_after();
          const uint32_t ahi = smem_u32(a_tile(s)), alo = smem_u32(alo_tile(s));
          const uint32_t bhi = smem_u32(bhi_tile(s)), blo = smem_u32(blo_tile(s));
          const uint32_t empty_peer = cluster_addr(&empty[s], peer);
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < BK / 8; ++j) {  // K = 8 tf32 (32 bytes) per MMA
              const uint32_t off = (uint32_t)j * 32u;
              const uint64_t dbh = smem_desc_sw<BK>(bhi + off), dbl = smem_desc_sw<BK>(blo + off);
              const uint64_t dah = smem_desc_sw<BK>(ahi + off), dal = smem_desc_sw<BK>(alo + off);
              umma2_tf32(d, dah, dbh, idesc, (kb > kb0 || j > 0) ? 1u : 0u);
              umma2_tf32(d, dah, dbl, idesc, 1u);
              umma2_tf32(d, dal, dbh, idesc, 1u);
            }
            umma2_commit(smem_u32(&empty[s]));
            umma2_commit(empty_peer);
          }
          __syncwarp();
        }
        if (ok) {
          const uint32_t accf_peer = cluster_addr(&accf[buf], peer);
          if (elect_one()) {
            umma2_commit(smem_u32(&accf[buf]));
            umma2_commit(accf_peer);
          }
          __syncwarp();
        }
      }
      if (!ok) {
        // every MMA issued so far retires before this arrives; wait for it
        // even though the pair is aborting, so neither CTA releases shared
        // memory or TMEM under them
        if (elect_one()) umma2_commit(smem_u32(drain));
        __syncwarp();
        pair_wait_warp(drain, 0, abort_flag, peer_abort, p.err, 5, /*ignore_abort=*/true);
      }
    }
  } else if (warp < 6) {
    // warps 2..5: split this CTA's A rows into tf32 hi (in place) and lo
    const int t128 = threadIdx.x - 64;
    uint32_t it = 0;
    bool ok = true;
    for (int u = pair; u < work.units && ok; u += npairs) {
      int m0, n0, width, kb0, kb1, slice;
      work.unit(u, BN, m0, n0, width, kb0, kb1, slice);
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        if (!(ok = pair_wait_warp(&full[s], (it / STAGES) & 1u, abort_flag, peer_abort, p.err, 6))) break;
        tc_split_a<(kTcBM * BK / 4) / 128>(reinterpret_cast<float4*>(a_tile(s)),
                                           reinterpret_cast<float4*>(alo_tile(s)), t128);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(cluster_addr(&conv[s], 0));
      }
    }
  } else {
    // warps 6..9: epilogue of this CTA's 128 rows, one TMEM lane quarter each
    const int q = warp & 3;
    if (lane == 0 && p.y_tma)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_y)) : "memory");
    const TcEpiSmem e = tc_epi_setup(p, epi_stage, warp - 6, head_smem);
    uint32_t tc = 0;
    for (int u = pair; u < work.units; u += npairs, ++tc) {
      const uint32_t buf = tc % NACC, use = tc / NACC;
      if (!pair_wait_warp(&accf[buf], use & 1u, abort_flag, peer_abort, p.err, 7)) break;
      tc_fence_after();
      int m0, n0, width, kb0, kb1, slice;
      work.unit(u, BN, m0, n0, width, kb0, kb1, slice);
      m0 += (int)rank * kTcBM;
      // split-K units store raw sums into their slice; the reduction applies the epilogue
      tc_epilogue_block<BN>(p, &map_y, e, tmem + buf * (uint32_t)BN + ((uint32_t)(q * 32) << 16), m0, n0, width, q,
                            lane, work.ksplit > 1 ? 0u : p.epi, slice);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&acce[buf], 0));
    }
    if (lane == 0) bulk_wait_all();  // this warp's output stores are complete before the CTA leaves
  }
  tc_fence_before();
  cluster_sync_all();  // no MMA of the pair and no remote arrival is still in flight
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// Shared-memory attribute and co-resident pair count, per device.
template <int BN, int BK, int STAGES>
inline int tc_pair_prepare(int* max_pairs) {
  using L = TcPairSmem<BN, BK, STAGES>;
  static std::atomic<int> cached[64];  // 0 = not yet, > 0 = pairs
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  if (cached[dev].load() > 0) {
    *max_pairs = cached[dev].load();
    return 0;
  }
  if (cudaFuncSetAttribute(tc_pair_gemm_kernel<BN, BK, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           L::TOTAL) != cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = L::TOTAL;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc_pair_gemm_kernel<BN, BK, STAGES>, &cfg) != cudaSuccess || n <= 0)
    return -1;
  cached[dev].store(n);
  *max_pairs = n;
  return 0;
}

// Returns 0 when launched, 1 when this GEMM cannot take this path, -1 on a
// launch error.
template <int BN, int BK, int STAGES>
inline int launch_tc_pair_bn(const TcArgs& t, const TcWeights& w, int* err, cudaStream_t s, bool ksplit_ok) {
  using L = TcPairSmem<BN, BK, STAGES>;
  int max_pairs = 0;
  if (tc_pair_prepare<BN, BK, STAGES>(&max_pairs) != 0) return -1;
  CUtensorMap map_a;
  if (!make_map_2d(&map_a, t.A, t.M, t.K, t.K, kTcBM, BK)) return 1;
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
  // TMA-store epilogue when the output rows are 16-byte aligned (no head:
  // then only the head's small outputs are written)
  CUtensorMap map_y;
  std::memset(&map_y, 0, sizeof(map_y));
  p.y_tma = (t.head.n == 0 && make_map_3d_out(&map_y, t.Y, 1, t.M, t.N)) ? 1 : 0;
  p.ksplit = 1;
  p.kb_per = 0;
  if (p.epi & EPI_BIAS_FIRST) p.epi = (p.epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
  if (p.head.epi & EPI_BIAS_FIRST) p.head.epi = (p.head.epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
  if (p.head.n > 0 && (t.N > BN || p.head.n > kTcMaxHeadN || t.N > kTcMaxHeadK)) return 1;
  const int64_t ntiles = ((t.M + 255) / 256) * ((t.N + BN - 1) / BN);
  // split-K when asked (ksplit_ok), the whole tiles cannot occupy half the
  // pairs and K is long (32 k-blocks or more: on shorter K the reduction pass
  // and the shorter pipelines cost more than the extra pairs give, measured
  // on 784- and 512-deep layers): S k-ranges per tile of at least 8 k-blocks
  // each, at most 16, their partial sums fitting the workspace, reduced in
  // slice order
  const int nk = (int)((t.K + BK - 1) / BK);
  const bool y_ok = (t.N * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(t.Y) & 15) == 0;
  const bool wants_ksplit = ksplit_ok && y_ok && t.ws && ntiles * 2 <= max_pairs && nk >= 32;
  // a fused head needs whole rows: when the shape wants split-K, decline the
  // fused form (the caller then runs the GEMM with split-K and the head as its
  // own step, much cheaper than one tile walking the whole K)
  if (wants_ksplit && t.head.n > 0) return 1;
  if (wants_ksplit && p.y_tma) {
    int S = (int)std::min<int64_t>(std::min<int64_t>(max_pairs / ntiles, nk / 8), 16);
    while (S > 1 && (size_t)S * (size_t)t.M * (size_t)t.N > t.ws_floats) --S;
    if (S > 1) {
      const int kb_per = (nk + S - 1) / S;
      S = (nk + kb_per - 1) / kb_per;  // no empty ranges
      CUtensorMap map_ws;
      if (S > 1 && make_map_3d_out(&map_ws, t.ws, S, t.M, t.N)) {
        p.ksplit = S;
        p.kb_per = kb_per;
        p.split = 1;
        p.split_from = (int)ntiles;
        const unsigned pairs = (unsigned)std::min<int64_t>(ntiles * S, max_pairs);
        if (pdl_launch(tc_pair_gemm_kernel<BN, BK, STAGES>, dim3(2 * pairs), dim3(kTcThreads), L::TOTAL, s, map_a,
                       w.map_hi[tc_bk_index(BK)][tc_bn_index(BN / 2)],
                       w.map_lo[tc_bk_index(BK)][tc_bn_index(BN / 2)], map_ws, p) != cudaSuccess)
          return -1;
        const int64_t quads = t.M * (t.N / 4);
        const int grid = (int)std::min<int64_t>(std::max<int64_t>((quads + 255) / 256, 1), (int64_t)max_pairs * 16);
        tc_splitk_reduce_kernel<<<grid, 256, 0, s>>>(t.ws, S, (int)t.M, (int)t.N, p.epi, p.bias, p.res, p.Y);
        return note_launch(cudaGetLastError());
      }
    }
  }
  // the last, partial round of tiles: cut into the slice count (1, 2 or 4,
  // slices at least 32 columns wide) that ends it soonest; not with a fused
  // head, which needs whole rows
  const int64_t rem = ntiles % max_pairs;
  int split = 1;
  if (rem > 0 && p.head.n == 0) {
    double best = 1.0;
    for (int f = 2; f <= 4 && BN / f >= 32; f *= 2) {
      const double rounds = (double)((f * rem + max_pairs - 1) / max_pairs) / f;
      if (rounds < best) best = rounds, split = f;
    }
  }
  p.split = split;
  p.split_from = (int)(ntiles - (split > 1 ? rem : 0));
  const int64_t units = p.split_from + (ntiles - p.split_from) * split;
  const unsigned pairs = (unsigned)std::min<int64_t>(units, max_pairs);
  // W^T maps with boxes of BN/2 rows: each CTA loads its half
  const int bi = tc_bn_index(BN / 2);
  const int ki = BK == 32 ? 0 : 1;
  return pdl_launch(tc_pair_gemm_kernel<BN, BK, STAGES>, dim3(2 * pairs), dim3(kTcThreads), L::TOTAL, s, map_a,
                    w.map_hi[ki][bi], w.map_lo[ki][bi], map_y, p) == cudaSuccess
             ? 0
             : -1;
}

// Tile configuration of one tensor-core launch: tile width BN and k-block BK.
// 0 picks by shape.  Stages fill the shared memory: k-blocks of 16 (64-byte
// swizzle) give twice the stages of 32.
struct TcConfig {
  int bn = 0;    // 64, 128 or 256
  int bk = 0;    // 16 or 32
  int mh = 0;    // one-SM tile rows: 1 -> 128, 2 -> 256 (two M=128 MMAs share each W k-block)
  int pair = 0;  // 1 = one SM per tile, 2 = 256-row tiles on an SM pair (BN 128 or 256),
                 // 3 = SM pair, split-K when the tiles cannot occupy the pairs
};

inline int launch_tc_gemm(const TcArgs& t, const TcWeights& w, int* err, int sm_count, cudaStream_t s,
                          TcConfig cfg = TcConfig{}) {
  if (!w.maps_ready || t.M <= 0) return 1;
  if (t.M > 0x7fffffff / 2 || t.N > 65535 * 64) return 1;
  const int bn = cfg.bn ? cfg.bn : tc_choose_bn(t.M, t.N, sm_count, t.head.n > 0);
  // 256-row tiles on SM pairs for tiles of 128 or 256 columns: they move a
  // third less operand data per MMA through shared memory, and when there
  // are fewer tiles than pairs the last round's column slices spread them
  // over more SMs than one-SM tiles would use
  const int64_t pair_tiles = ((t.M + 255) / 256) * ((t.N + bn - 1) / bn);
  const bool pair = cfg.pair >= 2 || (cfg.pair == 0 && cfg.mh != 2 && bn >= 128);
  // split-K (a different summation order) only where the caller allows it:
  // the shape rules (0) and the explicit SM-pair-with-split-K choice (3)
  const bool ksplit_ok = cfg.pair == 0 || cfg.pair == 3;
  // k-blocks of 32 when the tiles do not fill the pairs (fewer, larger stages
  // per tile) or K is long (measured on 4096/8192-deep layers: the per-k-block
  // overheads matter more than ring depth), 16 (deeper ring) otherwise
  const int bk = cfg.bk ? cfg.bk : (pair && (pair_tiles < sm_count / 2 || t.K >= 4096) ? 32 : 16);
  if (pair && bn >= 128) {
    if (bk == 32)
      return bn == 128 ? launch_tc_pair_bn<128, 32, 4>(t, w, err, s, ksplit_ok)
                       : launch_tc_pair_bn<256, 32, 3>(t, w, err, s, ksplit_ok);
    return bn == 128 ? launch_tc_pair_bn<128, 16, 8>(t, w, err, s, ksplit_ok)
                     : launch_tc_pair_bn<256, 16, 6>(t, w, err, s, ksplit_ok);
  }
  const int mh = (cfg.mh == 2 && bn <= 128) ? 2 : 1;
  if (mh == 2) {
    if (bk == 32) return bn == 64 ? launch_tc_bn<64, 32, 2, 2>(t, w, err, sm_count, s)
                                   : launch_tc_bn<128, 32, 2, 2>(t, w, err, sm_count, s);
    return bn == 64 ? launch_tc_bn<64, 16, 4, 2>(t, w, err, sm_count, s)
                    : launch_tc_bn<128, 16, 4, 2>(t, w, err, sm_count, s);
  }
  if (bk == 32) {
    switch (bn) {
      case 64: return launch_tc_bn<64, 32, 4, 1>(t, w, err, sm_count, s);
      case 128: return launch_tc_bn<128, 32, 3, 1>(t, w, err, sm_count, s);
      default: return launch_tc_bn<256, 32, 2, 1>(t, w, err, sm_count, s);
    }
  }
  switch (bn) {
    case 64: return launch_tc_bn<64, 16, 8, 1>(t, w, err, sm_count, s);
    case 128: return launch_tc_bn<128, 16, 6, 1>(t, w, err, sm_count, s);
    default: return launch_tc_bn<256, 16, 4, 1>(t, w, err, sm_count, s);
  }
}

}  // namespace ftb
