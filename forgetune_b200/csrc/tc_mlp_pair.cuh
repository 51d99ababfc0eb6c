// Two consecutive Linear layers in one kernel on SM pairs:
//
//   h = epi1(x W1),  y = epi2(h W2)  [and, with a head, y3 = epi3(y W3)]
//
// with h never leaving the chip.  The arithmetic is the SM-pair kernel's
// (tc_pair_gemm.cuh: 3xTF32 split, fp32 accumulation in TMEM, the same k
// order and the same epilogue operations), so the outputs are bit-identical
// to running the two layers as two launches.
//
// Per 256-row tile (two CTAs, 128 rows each):
//   layer 1   the SM-pair main loop (k-blocks of 16, W1^T halves of 128
//             rows) into TMEM columns [0, 256);
//   convert   the epilogue warps read h 32 columns at a time, apply the
//             layer-1 epilogue, split each value into tf32 hi and lo (what
//             the next layer's converter would do after loading h), write
//             hi back in place and lo into a four-slot ring of TMEM columns
//             [384, 512);
//   layer 2   tcgen05.mma with A read from TMEM (hi and lo) and W2^T halves
//             of 64 rows streamed through the same shared-memory ring as
//             layer 1's operands, into TMEM columns [256, 384);
//   epilogue  layer 2's epilogue (and the fused head) as in the SM-pair
//             kernel, overlapping the next tile's layer 1.
// The h tile (256 x N1 fp32) is never stored or re-read, and the two layers
// share one launch.
//
// Few tiles (a tile count that leaves at least one idle pair per tile): a
// team of S = 2 pairs computes one tile.  Many tiles whose last round would
// leave at least half of the pairs idle: the full rounds run unsplit and the
// tiles of the last round by teams (team.split_from = the first of them), so
// that round takes half of a tile's layer 1 instead of all of it.  Member s runs layer 1 over its own
// contiguous half of the k-blocks only; the helper (s = 1) writes its raw
// layer-1 sums (this CTA's 128 rows x 256 columns) to a workspace and bumps
// the tile's per-CTA counter; the owner (s = 0) waits for it (bounded), adds
// the helper's sums to its own while converting h (each chunk's sums loaded
// while the previous chunk is converted), and alone runs layer 2 and the
// head.  (Teams of more pairs were slower: the owner's added L2 round trips
// per chunk outweighed the shorter layer 1.)  The k terms are then
// associated differently from the unsplit kernel (deterministic, not the
// same bits).  Every CTA counts itself out at the end; the last one resets
// the counters, so each launch starts from zero, also after a wait that gave
// up.
//
// Hazards on TMEM: layer 1 of the next tile overwrites columns [0, 256)
// after layer 2 of this tile read its hi values there -- the MMAs of one
// thread run in issue order, and the MMA warp issues that layer 1 only after
// every chunk of this tile was converted.  A lo slot is rewritten only after
// the MMAs that read it have completed (lofree), layer 2's accumulator only
// after the epilogue drained it (acce2).
#pragma once

#include "tc_pair_gemm.cuh"

namespace ftb {

#define FTB_TMEM_ST32(taddr, r)                                                                                 \
  asm volatile(                                                                                                 \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17," \
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                             \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),         \
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), \
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),           \
      "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])                                   \
      : "memory")

// tcgen05.wait::ld for a load into r issued earlier: r is an operand, so the
// compiler treats the registers as written here (the load fills them
// asynchronously) and neither reads nor moves them before
#define FTB_TMEM_WAIT_LD32(r)                                                                                 \
  asm volatile("tcgen05.wait::ld.sync.aligned;"                                                               \
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), \
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),        \
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),      \
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),      \
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])                                                          \
               :                                                                                               \
               : "memory")

// D[256 x N] (+)= A[256 x 8] B[8 x N] over the SM pair, A (tf32) in the TMEM
// of both CTAs (lane = row, 8 columns from column a_tmem), B from shared
// memory.
__device__ __forceinline__ void umma2_tf32_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                                  uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// One chunk of h (32 columns of a row) from layer 1's accumulator to the
// tf32 hi / lo parts of layer 2's A operand, for the epilogues this kernel
// takes (a column bias and / or ReLU, fixed at compile time): per value
// v = relu(acc + b), hi = tf32(v), lo = tf32(v - hi), the operations of the
// layer-1 epilogue and the layer-2 converter (ReLU before and after a
// missing residual is ReLU once).
template <bool BIAS, bool RELU>
__device__ __forceinline__ void mlp_split_chunk(const uint32_t (&r)[32], const float* b, uint32_t (&hi)[32],
                                                uint32_t (&lo)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 bb = BIAS ? reinterpret_cast<const float4*>(b)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    const float b4[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float v = __uint_as_float(r[4 * i + k]);
      if (BIAS) v = __fadd_rn(v, b4[k]);
      if (RELU) v = relu_keep_nan(v);
      const float h = tf32_rna(v);
      hi[4 * i + k] = __float_as_uint(h);
      lo[4 * i + k] = __float_as_uint(tf32_rna_rem(v - h));
    }
  }
}

// The team helper's raw sums of one chunk (32 floats of a row: float4
// group i at src[i * 128], rows adjacent), loaded ahead of their use, and
// added to r.
__device__ __forceinline__ void mlp_load_partial(float4 (&v4)[8], const float4* src) {
#pragma unroll
  for (int i = 0; i < 8; ++i) v4[i] = __ldcg(src + i * 128);
}
__device__ __forceinline__ void mlp_add_partial(uint32_t (&r)[32], const float4 (&v4)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    r[4 * i + 0] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * i + 0]), v4[i].x));
    r[4 * i + 1] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * i + 1]), v4[i].y));
    r[4 * i + 2] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * i + 2]), v4[i].z));
    r[4 * i + 3] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * i + 3]), v4[i].w));
  }
}

constexpr int kTcMlpN1 = 256;  // layer 1's width: its accumulator is TMEM columns [0, 256)
constexpr int kTcMlpN2 = 128;  // layer 2's width: columns [256, 384)

template <int STAGES>
struct TcMlpSmem {
  static constexpr int A_BYTES = kTcBM * 16 * 4;        // this CTA's 128 rows of a 16-wide k-block of x
  static constexpr int B_BYTES = 128 * 16 * 4;          // this CTA's half of a W1^T k-block
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TX1 = A_BYTES + 2 * B_BYTES;      // a layer-1 stage
  static constexpr int TX2 = 2 * 64 * 16 * 4;            // a layer-2 stage: 64 rows of W2^T, hi and lo
  static constexpr int EPI_BYTES = 4 * 32 * 33 * 4;
  static constexpr int HEAD_BYTES = (kTcMaxHeadK * kTcMaxHeadN + kTcMaxHeadK + kTcMaxHeadN) * 4;
  static constexpr int NBAR = 3 * STAGES + 13;
  static constexpr int BAR_BYTES = 8 * NBAR + 16;
  static constexpr int TOTAL = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + HEAD_BYTES + BAR_BYTES;
};

// The small head over layer 2's columns [c0, c1) of this warp's rows, the
// layer-2 epilogue applied per value on the way (head_chunk of tc_gemm.cuh):
// partial sums of the head's outputs, in column order from zero.  Every
// lane computes, rows past M too (finite values of zero-filled input rows,
// never stored; this kernel's epilogues read no [M, N] operand), so the
// loop does not diverge: 1.9 us less per launch at 8192 rows than with the
// rows past M skipped.
template <int HP4>
__device__ __forceinline__ void mlp_head_part(float (&acc)[4 * HP4], const TcKernelParams& p2, const TcEpiSmem& e,
                                              uint32_t base, int m, int c0, int c1) {
#pragma unroll
  for (int o = 0; o < 4 * HP4; ++o) acc[o] = 0.0f;
#pragma unroll 1
  for (int c = c0; c < c1; c += 32) {
    uint32_t r[32];
    __syncwarp();
    FTB_TMEM_LD32(base + (uint32_t)c, r);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    const int cnt = min(32, c1 - c);
    if (cnt == 32)
      head_chunk<HP4, true, false>(acc, r, p2, e, m, c, cnt);
    else
      head_chunk<HP4, false, false>(acc, r, p2, e, m, c, cnt);
  }
}

// The head after layer 2 when a pair computes a single tile (and the launch
// allows a different association of the head's sums than the sequential one
// of two launches: by shape or pair 5): eight warps
// share it -- the epilogue warps (grp 0) take layer 2's columns [0, 64), the
// split warps (grp 1, idle once layer 1 is done) the rest -- and the epilogue
// warps add the split warps' partial sums (staged in `part`, 128 rows x 16)
// to theirs and store the outputs.  Every thread of both groups passes both
// named barriers (id 3), also after an abort.
template <int HP4>
__device__ __forceinline__ void mlp_head_shared(const TcKernelParams& p2, const TcEpiSmem& e, uint32_t base, int m,
                                                int row, int grp, bool ok, float* part) {
  float acc[4 * HP4];
  const int n2 = p2.N;
  const int c0 = grp == 0 ? 0 : 64, c1 = grp == 0 ? min(64, n2) : n2;
  asm volatile("bar.sync 3, 256;" ::: "memory");
  if (ok && c0 < c1) {
    mlp_head_part<HP4>(acc, p2, e, base, m, c0, c1);
  } else {
#pragma unroll
    for (int o = 0; o < 4 * HP4; ++o) acc[o] = 0.0f;
  }
  if (grp == 1) {
#pragma unroll
    for (int o = 0; o < 4 * HP4; ++o) part[row * 16 + o] = acc[o];
  }
  asm volatile("bar.sync 3, 256;" ::: "memory");
  if (grp == 0 && ok && m < p2.M) {
#pragma unroll
    for (int o = 0; o < 4 * HP4; ++o) {
      if (o < e.hn) {
        const float v = __fadd_rn(acc[o], part[row * 16 + o]);
        p2.head.y[(int64_t)m * e.hn + o] = apply_epilogue(v, p2.head.epi, e.head_bb, nullptr, m, o, e.hn);
      }
    }
  }
}

__device__ __forceinline__ void mlp_head_dispatch(const TcKernelParams& p2, const TcEpiSmem& e, uint32_t base, int m,
                                                  int row, int grp, bool ok, float* part) {
  switch (e.hp) {
    case 4: mlp_head_shared<1>(p2, e, base, m, row, grp, ok, part); break;
    case 8: mlp_head_shared<2>(p2, e, base, m, row, grp, ok, part); break;
    case 12: mlp_head_shared<3>(p2, e, base, m, row, grp, ok, part); break;
    default: mlp_head_shared<4>(p2, e, base, m, row, grp, ok, part); break;
  }
}

// Split of layer 1 over a team of pairs (S = 1: no split).
struct TcMlpTeam {
  float* ws;         // helper sums: per tile and CTA rank 128 rows x 256 columns, as [chunk][group of 4][row] float4s
  unsigned* flags;   // [tile][CTA rank][group of four chunks]: helper warps that published those sums
  unsigned* depart;  // CTAs that left the launch
  int S;
  int share_head;  // a pair with a single tile shares the head between its warp groups
  int split_from;  // the first tile computed by a team (0: all of them)
};

constexpr int kTcMlpMaxTeam = 2;
constexpr int kTcMlpMaxChunks = 8;  // 32-column chunks of h (N1 <= 256)
constexpr int kTcMlpFlagStride = 32;  // counter words per (tile, CTA rank): one 128-byte line each

// Bounded wait (one thread) until *f reaches `want`; on timeout it raises
// this CTA's and the peer's abort flags and records error code 10.
__device__ __forceinline__ int team_wait(const unsigned* f, unsigned want, volatile int* abort_flag,
                                         uint32_t peer_abort, int* err) {
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v >= want) return 1;
    __nanosleep(64);
    if ((it & 63u) == 63u) {
      if (*abort_flag) return 0;
      if (global_ns() - t0 > kTcWaitLimitNs) {
        *abort_flag = 1;
        st_cluster_u32(peer_abort, 1u);
        atomicCAS(err, 0, 10);
        return 0;
      }
    }
  }
}
constexpr int kTcMlpTeamFlagWords = 2400;  // [tile][CTA rank] lines of chunk counters (2 x 37 x 32) + the departure counter

// p1: layer 1 (M, K = K1, N = N1, bias, epi); p2: layer 2 (K = N1, N = N2,
// bias, epi, output Y / head).  Roles as in the SM-pair kernel; the
// epilogue warps also convert h.
template <int STAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    tc_mlp_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w1hi,
                       const __grid_constant__ CUtensorMap map_w1lo, const __grid_constant__ CUtensorMap map_w2hi,
                       const __grid_constant__ CUtensorMap map_w2lo, const __grid_constant__ CUtensorMap map_y,
                       TcKernelParams p1, TcKernelParams p2, TcMlpTeam team) {
  using L = TcMlpSmem<STAGES>;
  static_assert(L::TOTAL <= 227 * 1024, "shared memory budget");
  constexpr uint32_t TMEM_COLS = 512, ACC2 = 256, LO = 384;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  auto a_tile = [&](int s) { return reinterpret_cast<float*>(smem + s * L::STAGE_BYTES); };
  auto alo_tile = [&](int s) { return reinterpret_cast<float*>(smem + s * L::STAGE_BYTES + L::A_BYTES); };
  auto bhi_tile = [&](int s) { return smem + s * L::STAGE_BYTES + 2 * L::A_BYTES; };
  auto blo_tile = [&](int s) { return smem + s * L::STAGE_BYTES + 2 * L::A_BYTES + L::B_BYTES; };
  float* epi_stage = reinterpret_cast<float*>(smem + STAGES * L::STAGE_BYTES);
  float* head_smem = reinterpret_cast<float*>(smem + STAGES * L::STAGE_BYTES + L::EPI_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * L::STAGE_BYTES + L::EPI_BYTES + L::HEAD_BYTES);
  uint64_t* full = bars;                // this CTA's TMA landed
  uint64_t* conv = bars + STAGES;       // leader: stage ready in both CTAs (8 arrivals)
  uint64_t* empty = bars + 2 * STAGES;  // the pair's MMAs done reading the stage
  uint64_t* accf1 = bars + 3 * STAGES;  // layer 1's accumulator complete
  uint64_t* accf2 = accf1 + 1;          // layer 2's accumulator complete
  uint64_t* acce2 = accf2 + 1;          // leader: layer 2's accumulator drained (8 arrivals)
  uint64_t* a2rdy = acce2 + 1;          // [4] leader: a chunk of h converted in both CTAs (8 arrivals)
  uint64_t* lofree = a2rdy + 4;         // [4] the MMAs reading a lo slot completed
  uint64_t* drain = lofree + 4;         // leader: MMAs retired after an abort
  uint64_t* never = drain + 1;          // never arrived on (stall_test)
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(never + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(never + 1) + 1;

  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles = (p1.M + 255) / 256;
  const int nk1 = (p1.K + 15) / 16;
  const int nk2 = (p1.N + 15) / 16;  // layer 2's k-blocks (K2 = N1)
  const int nch = (p1.N + 31) / 32;  // chunks of h converted per tile
  const int pair = (int)cluster_index();
  const int npairs = (int)cluster_count();
  // this pair's tiles: p, p + npairs, ... below split_from with all of layer
  // 1's k-blocks; the tiles from split_from on (all of them when they are
  // few, the last round when they are many) are shared by teams of S pairs:
  // pair p < S x Lt is member p / Lt of tile split_from + p % Lt, with the
  // member's contiguous share of the k-blocks; member 0 (the owner) also runs
  // layer 2 and the head
  const int S = team.S;
  const bool teamed = S > 1;  // the launch splits some tiles
  const int split_from = teamed ? team.split_from : tiles;
  const int Lt = tiles - split_from;  // tiles computed by teams
  const int team_u = (teamed && Lt > 0 && pair < S * Lt) ? split_from + pair % Lt : tiles;
  const int member = (teamed && Lt > 0) ? pair / Lt : 0;
  const int u_first = pair < split_from ? pair : team_u;
  auto u_next = [&](int u) { return u + npairs < split_from ? u + npairs : (u < split_from ? team_u : tiles); };
  auto in_team = [&](int u) { return u >= split_from; };
  auto owner_of = [&](int u) { return !in_team(u) || member == 0; };
  auto kb_lo_of = [&](int u) { return in_team(u) ? (member * nk1) / S : 0; };
  auto kb_hi_of = [&](int u) { return in_team(u) ? ((member + 1) * nk1) / S : nk1; };
  // one tile for this pair and a head after layer 2: the split warps share
  // the head (they are idle once layer 1 is done)
  const bool head_shared =
      team.share_head && u_first < tiles && owner_of(u_first) && p2.head.n > 0 && u_next(u_first) >= tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 8);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf1, 1);
    mbar_init(accf2, 1);
    mbar_init(acce2, 8);
    for (int q = 0; q < 4; ++q) {
      mbar_init(&a2rdy[q], 8);
      mbar_init(&lofree[q], 1);
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
  cluster_sync_all();
  tc_fence_after();
  grid_dep_wait();
  grid_dep_trigger();
  const uint32_t tmem = *tmem_slot;
  const uint32_t peer_abort = cluster_addr(const_cast<int*>(abort_flag), peer);

  if (warp == 0) {
    if (lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    const uint64_t pol_a = l2_evict_first();  // x is read once
    const uint64_t pol_w = l2_evict_last();   // both weights are re-read by every tile
    uint32_t it = 0;
    bool ok = true;
    for (int u = u_first; u < tiles && ok; u = u_next(u)) {
      const int m0 = u * 256 + (int)rank * kTcBM;
      const int kb_hi = kb_hi_of(u);
      for (int kb = kb_lo_of(u); kb < kb_hi; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        if (!(ok = pair_wait_warp(&empty[s], ((it / STAGES) & 1u) ^ 1u, abort_flag, peer_abort, p1.err, 1))) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full[s], L::TX1);
          tma_load_2d_hint(a_tile(s), &map_a, kb * 16, m0, &full[s], pol_a);
          tma_load_2d_hint(bhi_tile(s), &map_w1hi, kb * 16, (int)rank * 128, &full[s], pol_w);
          tma_load_2d_hint(blo_tile(s), &map_w1lo, kb * 16, (int)rank * 128, &full[s], pol_w);
        }
        __syncwarp();
      }
      for (int j = 0; j < nk2 && ok && owner_of(u); ++j, ++it) {
        const int s = (int)(it % STAGES);
        if (!(ok = pair_wait_warp(&empty[s], ((it / STAGES) & 1u) ^ 1u, abort_flag, peer_abort, p1.err, 1))) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full[s], L::TX2);
          tma_load_2d_hint(bhi_tile(s), &map_w2hi, j * 16, (int)rank * 64, &full[s], pol_w);
          tma_load_2d_hint(blo_tile(s), &map_w2lo, j * 16, (int)rank * 64, &full[s], pol_w);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      uint32_t it = 0, tc = 0, g = 0;
      bool ok = true;
      if (p1.stall_test) ok = pair_wait_warp(never, 0, abort_flag, peer_abort, p1.err, 9);
      const uint32_t idesc1 = idesc_tf32_pair(256), idesc2 = idesc_tf32_pair(kTcMlpN2);
      for (int u = u_first; u < tiles && ok; u = u_next(u), ++tc) {
        // layer 1 into columns [0, 256); this tile's layer 2 of the previous
        // tile, issued earlier, has read its A there first
        const int kb_lo = kb_lo_of(u), kb_hi = kb_hi_of(u);
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
          const int s = (int)(it % STAGES);
          if (!(ok = pair_wait_warp(&conv[s], (it / STAGES) & 1u, abort_flag, peer_abort, p1.err, 4))) break;
          tc_fence_after();
          const uint32_t ahi = smem_u32(a_tile(s)), alo = smem_u32(alo_tile(s));
          const uint32_t bhi = smem_u32(bhi_tile(s)), blo = smem_u32(blo_tile(s));
          const uint32_t empty_peer = cluster_addr(&empty[s], peer);
          if (elect_one()) {
#pragma unroll
            for (int k8 = 0; k8 < 2; ++k8) {
              const uint32_t off = (uint32_t)k8 * 32u;
              const uint64_t dbh = smem_desc_sw<16>(bhi + off), dbl = smem_desc_sw<16>(blo + off);
              const uint64_t dah = smem_desc_sw<16>(ahi + off), dal = smem_desc_sw<16>(alo + off);
              umma2_tf32(tmem, dah, dbh, idesc1, (kb > kb_lo || k8 > 0) ? 1u : 0u);
              umma2_tf32(tmem, dah, dbl, idesc1, 1u);
              umma2_tf32(tmem, dal, dbh, idesc1, 1u);
            }
            umma2_commit(smem_u32(&empty[s]));
            umma2_commit(empty_peer);
          }
          __syncwarp();
        }
        if (!ok) break;
        {
          const uint32_t peer_bar = cluster_addr(accf1, peer);
          if (elect_one()) {
            umma2_commit(smem_u32(accf1));
            umma2_commit(peer_bar);
          }
          __syncwarp();
        }
        if (!owner_of(u)) continue;  // a helper's part ends with its layer-1 sums
        // layer 2 into columns [256, 384), once the previous tile's epilogue drained them
        if (!(ok = pair_wait_warp(acce2, (tc & 1u) ^ 1u, abort_flag, peer_abort, p1.err, 2))) break;
        tc_fence_after();
        for (int j = 0; j < nk2; ++j, ++it) {
          const int s = (int)(it % STAGES);
          const uint32_t gc = g + (uint32_t)(j >> 1);  // chunk of h
          const uint32_t q = gc & 3u;
          if ((j & 1) == 0) {
            if (!(ok = pair_wait_warp(&a2rdy[q], (gc >> 2) & 1u, abort_flag, peer_abort, p1.err, 3))) break;
            tc_fence_after();
          }
          if (!(ok = pair_wait_warp(&conv[s], (it / STAGES) & 1u, abort_flag, peer_abort, p1.err, 4))) break;
          tc_fence_after();
          const uint32_t bhi = smem_u32(bhi_tile(s)), blo = smem_u32(blo_tile(s));
          const uint32_t empty_peer = cluster_addr(&empty[s], peer);
          const uint32_t lofree_peer = cluster_addr(&lofree[q], peer);
          const bool last_of_chunk = (j & 1) == 1 || j == nk2 - 1;
          if (elect_one()) {
#pragma unroll
            for (int k8 = 0; k8 < 2; ++k8) {
              const uint32_t off = (uint32_t)k8 * 32u;
              const uint64_t dbh = smem_desc_sw<16>(bhi + off), dbl = smem_desc_sw<16>(blo + off);
              const uint32_t ahi = tmem + (uint32_t)(16 * j + 8 * k8);
              const uint32_t alo = tmem + LO + 32u * q + (uint32_t)(16 * (j & 1) + 8 * k8);
              umma2_tf32_tmem_a(tmem + ACC2, ahi, dbh, idesc2, (j > 0 || k8 > 0) ? 1u : 0u);
              umma2_tf32_tmem_a(tmem + ACC2, ahi, dbl, idesc2, 1u);
              umma2_tf32_tmem_a(tmem + ACC2, alo, dbh, idesc2, 1u);
            }
            umma2_commit(smem_u32(&empty[s]));
            umma2_commit(empty_peer);
            if (last_of_chunk) {
              umma2_commit(smem_u32(&lofree[q]));
              umma2_commit(lofree_peer);
            }
          }
          __syncwarp();
        }
        g += (uint32_t)nch;
        if (!ok) break;
        {
          const uint32_t peer_bar = cluster_addr(accf2, peer);
          if (elect_one()) {
            umma2_commit(smem_u32(accf2));
            umma2_commit(peer_bar);
          }
          __syncwarp();
        }
      }
      if (!ok) {
        // every MMA issued so far retires before this arrives
        if (elect_one()) umma2_commit(smem_u32(drain));
        __syncwarp();
        pair_wait_warp(drain, 0, abort_flag, peer_abort, p1.err, 5, /*ignore_abort=*/true);
      }
    }
  } else if (warp < 6) {
    // warps 2..5: split layer 1's A rows into tf32 hi (in place) and lo; a
    // layer-2 stage (W2 only) is passed on once it has landed
    const int t128 = threadIdx.x - 64;
    uint32_t it = 0;
    bool ok = true;
    for (int u = u_first; u < tiles && ok; u = u_next(u)) {
      const int nkl = kb_hi_of(u) - kb_lo_of(u);
      for (int kb = 0; kb < nkl + (owner_of(u) ? nk2 : 0); ++kb, ++it) {
        const int s = (int)(it % STAGES);
        if (!(ok = pair_wait_warp(&full[s], (it / STAGES) & 1u, abort_flag, peer_abort, p1.err, 6))) break;
        if (kb < nkl) {
          tc_split_a<(kTcBM * 16 / 4) / 128>(reinterpret_cast<float4*>(a_tile(s)),
                                             reinterpret_cast<float4*>(alo_tile(s)), t128);
          fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(cluster_addr(&conv[s], 0));
      }
    }
    if (head_shared) {
      // the second half of layer 2's columns through the head
      const int qq = warp & 3;
      const int row = qq * 32 + lane;
      const int m = u_first * 256 + (int)rank * kTcBM + row;
      const bool okh = ok && pair_wait_warp(accf2, 0u, abort_flag, peer_abort, p1.err, 7);
      tc_fence_after();
      TcEpiSmem es;
      es.tr = nullptr;
      es.stage = nullptr;
      es.head_w = head_smem;  // staged by the epilogue warps (tc_epi_setup) at the start
      es.bias_a = head_smem + kTcMaxHeadK * kTcMaxHeadN;
      es.head_bb = es.bias_a + kTcMaxHeadK;
      es.hn = p2.head.n;
      es.hp = (es.hn + 3) & ~3;
      mlp_head_dispatch(p2, es, tmem + ACC2 + ((uint32_t)(qq * 32) << 16), m, row, 1, okh,
                        reinterpret_cast<float*>(a_tile(0)));
      tc_fence_before();
    }
  } else {
    // warps 6..9: convert h, then layer 2's epilogue, for this CTA's 128 rows
    // (one TMEM lane quarter each)
    const int q = warp & 3;
    const uint32_t lanes = (uint32_t)(q * 32) << 16;
    if (lane == 0 && p2.y_tma)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_y)) : "memory");
    const TcEpiSmem e = tc_epi_setup(p2, epi_stage, warp - 6, head_smem);
    // layer 1's column bias, zero past N1, in whichever area layer 2's
    // epilogue leaves unused (the head's with no head, the staging tiles'
    // with one)
    float* b1s = p2.head.n > 0 ? epi_stage : head_smem;
    const bool bias1 = p1.bias != nullptr && (p1.epi & EPI_BIAS_LAST);
    for (int i = threadIdx.x - 192; i < kTcMlpN1; i += 128) b1s[i] = (bias1 && i < p1.N) ? p1.bias[i] : 0.0f;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const uint32_t a2rdy_leader = cluster_addr(&a2rdy[0], 0);
    // layer 1's epilogue: a column bias and / or ReLU (tc_mlp_supported)
    const bool ep_bias = (p1.epi & EPI_BIAS_LAST) != 0;
    const bool ep_relu = (p1.epi & (EPI_RELU_PRE | EPI_RELU_POST)) != 0;
    uint32_t tc = 0, g = 0;
    bool ok = true;
    for (int u = u_first; u < tiles && ok; u = u_next(u), ++tc) {
      const int m0 = u * 256 + (int)rank * kTcBM;
      if (!(ok = pair_wait_warp(accf1, tc & 1u, abort_flag, peer_abort, p1.err, 7))) break;
      tc_fence_after();
      // chunk c+1 is loaded from TMEM while chunk c's stores complete
      uint32_t r[32];
      const int row = q * 32 + lane;  // this thread's row of the CTA's 128
      if (!owner_of(u)) {
        // helper: publish this CTA's raw layer-1 sums, then count them in
        // layout [chunk][float4 group][row] of float4s: a warp's store is 512
        // contiguous bytes (its 32 rows' group i), and so is the owner's load
        // (each warp counts its 32 rows of a chunk in as soon as they are stored)
        const int tu = u - split_from;  // this tile among the team tiles
        float4* dst = reinterpret_cast<float4*>(team.ws + (size_t)(tu * 2 + (int)rank) * 128 * 256) + row;
        unsigned* fl = team.flags + (2 * tu + (int)rank) * kTcMlpFlagStride;
        for (int c = 0; c < nch; ++c) {
          __syncwarp();
          FTB_TMEM_LD32(tmem + lanes + (uint32_t)(32 * c), r);
          FTB_TMEM_WAIT_LD32(r);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[(c * 8 + i) * 128] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                                 __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
          // each group of four chunks is published with one release (a
          // release waits for the warp's stores: one per chunk would stall
          // the loop an L2 round trip per chunk)
          if ((c & 3) == 3 || c + 1 == nch) {
            __syncwarp();
            if (lane == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(fl + (c >> 2)) : "memory");
          }
        }
        tc_fence_before();
        continue;
      }
      // the helper's sums of this thread's row (chunk c at 32 c), each chunk
      // loaded while the one before it is converted
      const bool tsum = in_team(u);  // the helper's sums are added to this tile's
      const int tu = tsum ? u - split_from : 0;
      const float4* hrow = reinterpret_cast<const float4*>(team.ws + (size_t)(tu * 2 + (int)rank) * 128 * 256) + row;
      const unsigned* hfl = team.flags + (2 * tu + (int)rank) * kTcMlpFlagStride;
      // the helper's four warps have stored chunk c of this CTA's rows (they
      // publish groups of four chunks; lane 0 waits, bounded; the warp then reads)
      auto chunk_ready = [&](int c) -> bool {
        if (c & 3) return true;  // published with the first chunk of its group of four
        int okc = 1;
        if (lane == 0) okc = team_wait(hfl + (c >> 2), 4u, abort_flag, peer_abort, p1.err);
        okc = __shfl_sync(0xffffffffu, okc, 0);
        __syncwarp();
        return okc != 0;
      };
      float4 pn[8];
      if (tsum) {
        if (!(ok = chunk_ready(0))) break;
        mlp_load_partial(pn, hrow);
      }
      __syncwarp();
      FTB_TMEM_LD32(tmem + lanes, r);
      FTB_TMEM_WAIT_LD32(r);
      for (int c = 0; c < nch; ++c) {
        const uint32_t gc = g + (uint32_t)c, qs = gc & 3u, use = gc >> 2;
        uint32_t hi[32], lo[32];
        if (tsum) {
          mlp_add_partial(r, pn);
          if (c + 1 < nch) {
            if (!(ok = chunk_ready(c + 1))) break;
            mlp_load_partial(pn, hrow + (c + 1) * 8 * 128);
          }
        }
        const float* b = b1s + 32 * c;
        if (ep_bias && ep_relu) mlp_split_chunk<true, true>(r, b, hi, lo);
        else if (ep_bias) mlp_split_chunk<true, false>(r, b, hi, lo);
        else if (ep_relu) mlp_split_chunk<false, true>(r, b, hi, lo);
        else mlp_split_chunk<false, false>(r, b, hi, lo);
        __syncwarp();
        if (c + 1 < nch) FTB_TMEM_LD32(tmem + lanes + (uint32_t)(32 * (c + 1)), r);
        FTB_TMEM_ST32(tmem + lanes + (uint32_t)(32 * c), hi);
        // the lo slot is free once the MMAs that read its previous chunk completed
        if (use >= 1) {
          if (!(ok = pair_wait_warp(&lofree[qs], (use - 1) & 1u, abort_flag, peer_abort, p1.err, 8))) break;
          tc_fence_after();
        }
        FTB_TMEM_ST32(tmem + lanes + LO + 32u * qs, lo);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(a2rdy_leader + 8u * qs);
        FTB_TMEM_WAIT_LD32(r);
      }
      FTB_TMEM_WAIT_LD32(r);  // nothing left in flight if the loop gave up
      g += (uint32_t)nch;
      if (!ok) break;
      if (head_shared) break;  // the head follows, shared with the split warps
      if (!(ok = pair_wait_warp(accf2, tc & 1u, abort_flag, peer_abort, p1.err, 7))) break;
      tc_fence_after();
      tc_epilogue_block<kTcMlpN2>(p2, &map_y, e, tmem + ACC2 + lanes, m0, 0, kTcMlpN2, q, lane, p2.epi, 0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(acce2, 0));
    }
    if (head_shared) {
      // the first half of layer 2's columns through the head, plus the split
      // warps' half, then the outputs
      const int row = q * 32 + lane;
      const int m = u_first * 256 + (int)rank * kTcBM + row;
      const bool okh = ok && pair_wait_warp(accf2, 0u, abort_flag, peer_abort, p1.err, 7);
      tc_fence_after();
      mlp_head_dispatch(p2, e, tmem + ACC2 + lanes, m, row, 0, okh, reinterpret_cast<float*>(a_tile(0)));
      tc_fence_before();
    }
    if (lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  cluster_sync_all();  // no MMA of the pair and no remote arrival is still in flight
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
  if (teamed) {
    // every role of this CTA is done: count it out; the last CTA out resets
    // the chunk counters (all threads, plain stores: the next launch sees
    // them once this one has completed)
    volatile int* last = reinterpret_cast<volatile int*>(never + 1) + 2;
    if (threadIdx.x == 0) {
      __threadfence();
      *last = atomicAdd(team.depart, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (*last) {
      for (int i = threadIdx.x; i < 2 * Lt * 2; i += blockDim.x) team.flags[(i >> 1) * kTcMlpFlagStride + (i & 1)] = 0u;
      if (threadIdx.x == 0) *team.depart = 0u;
    }
  }
}

// Shared-memory attribute and co-resident pair count, per device.
template <int STAGES>
inline int tc_mlp_prepare(int* max_pairs) {
  using L = TcMlpSmem<STAGES>;
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  if (cached[dev].load() > 0) {
    *max_pairs = cached[dev].load();
    return 0;
  }
  if (cudaFuncSetAttribute(tc_mlp_pair_kernel<STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL) !=
      cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = L::TOTAL;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc_mlp_pair_kernel<STAGES>, &cfg) != cudaSuccess || n <= 0) return -1;
  cached[dev].store(n);
  *max_pairs = n;
  return 0;
}

// Whether two Linear layers (t1 then t2, t2 reading only t1's output) fit
// the fused kernel: 128 < N1 <= 256, N2 <= 128, epilogues of a column bias
// and ReLUs (no [M, N] bias or residual), both weights in tensor-core layout.
inline bool tc_mlp_supported(const TcArgs& t1, const TcWeights& w1, const TcArgs& t2, const TcWeights& w2) {
  const uint32_t bad = EPI_BIAS_ROWS | EPI_RESIDUAL;
  const uint32_t epi1_ok = EPI_BIAS_FIRST | EPI_BIAS_LAST | EPI_RELU_PRE | EPI_RELU_POST;
  if (!w1.maps_ready || !w2.maps_ready) return false;
  if (t1.epi & ~epi1_ok) return false;
  if (t1.N <= 128 || t1.N > kTcMlpN1 || t2.K != t1.N || t2.N < 1 || t2.N > kTcMlpN2) return false;
  if ((t1.epi & bad) || (t2.epi & bad)) return false;
  if (t2.head.n > 0 && (t2.head.n > kTcMaxHeadN || t2.N > kTcMaxHeadK)) return false;
  if (t1.M <= 0 || t1.M > 0x7fffffff / 2 || t1.K > 0x7fffffff) return false;
  return true;
}

// Team size for `tiles` tiles of layer 1 with nk1 k-blocks: two pairs per
// tile when the tiles leave that many free, each member keeping at least
// eight k-blocks.
inline int tc_mlp_team_size(int64_t tiles, int nk1, int max_pairs) {
  if (tiles <= 0) return 1;
  int S = (int)std::min<int64_t>(kTcMlpMaxTeam, max_pairs / tiles);
  S = std::min(S, nk1 / 8);
  return S >= 2 ? S : 1;
}

// Returns 0 when launched, 1 when the pair of layers cannot take this path,
// -1 on a launch error.  With `team_flags` (kTcMlpTeamFlagWords zeroed words)
// and the split-K workspace in t1.ws, few tiles run split over teams of pairs.
inline int launch_tc_mlp(const TcArgs& t1, const TcWeights& w1, const TcArgs& t2, const TcWeights& w2, int* err,
                         cudaStream_t s, unsigned* team_flags = nullptr) {
  constexpr int STAGES = 6;
  using L = TcMlpSmem<STAGES>;
  if (!tc_mlp_supported(t1, w1, t2, w2)) return 1;
  int max_pairs = 0;
  if (tc_mlp_prepare<STAGES>(&max_pairs) != 0) return -1;
  CUtensorMap map_a;
  if (!make_map_2d(&map_a, t1.A, t1.M, t1.K, t1.K, kTcBM, 16)) return 1;
  auto params = [&](const TcArgs& t) {
    TcKernelParams p;
    std::memset(&p, 0, sizeof(p));
    p.bias = t.bias;
    p.res = nullptr;
    p.Y = t.Y;
    p.M = (int)t.M;
    p.N = (int)t.N;
    p.K = (int)t.K;
    p.epi = t.epi;
    p.head = t.head;
    p.err = err;
    p.stall_test = t.stall_test;
    p.split = 1;
    p.ksplit = 1;
    // the accumulators start at zero: a bias-first epilogue adds the bias at the end
    if (p.epi & EPI_BIAS_FIRST) p.epi = (p.epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
    if (p.head.epi & EPI_BIAS_FIRST) p.head.epi = (p.head.epi & ~(uint32_t)EPI_BIAS_FIRST) | EPI_BIAS_LAST;
    return p;
  };
  TcKernelParams p1 = params(t1), p2 = params(t2);
  p1.head = TcHead{};
  CUtensorMap map_y;
  std::memset(&map_y, 0, sizeof(map_y));
  p2.y_tma = (t2.head.n == 0 && make_map_3d_out(&map_y, t2.Y, 1, t2.M, t2.N)) ? 1 : 0;
  const int64_t tiles = (t1.M + 255) / 256;
  unsigned pairs = (unsigned)std::min<int64_t>(tiles, max_pairs);
  TcMlpTeam team;
  std::memset(&team, 0, sizeof(team));
  team.S = 1;
  if (team_flags && t1.ws) {
    // by shape or asked for (pair 5): the sums may be associated differently
    // from two launches -- layer 1 split over teams, the head shared
    team.share_head = 1;
    const int nk1 = (int)((t1.K + 15) / 16);
    int S = tc_mlp_team_size(tiles, nk1, max_pairs);
    int64_t split_from = 0, team_tiles = tiles;
    if (S == 1 && tiles > max_pairs) {
      // many tiles: the full rounds unsplit, a last round that leaves at
      // least half of the pairs idle split over teams
      const int64_t full = tiles / max_pairs * max_pairs;
      const int S_last = tc_mlp_team_size(tiles - full, nk1, max_pairs);
      if (tiles > full && S_last > 1) {
        S = S_last;
        split_from = full;
        team_tiles = tiles - full;
      }
    }
    const size_t need = (size_t)(S - 1) * (size_t)team_tiles * 2 * 128 * 256;
    if (S > 1 && need <= t1.ws_floats && 2 * team_tiles * kTcMlpFlagStride <= kTcMlpTeamFlagWords - 1) {
      team.S = S;
      team.split_from = (int)split_from;
      team.ws = t1.ws;
      team.flags = team_flags;
      team.depart = team_flags + kTcMlpTeamFlagWords - 1;
      pairs = split_from > 0 ? (unsigned)max_pairs : (unsigned)(tiles * S);
    }
  }
  // W1^T halves of 128 rows, W2^T halves of 64 rows, k-blocks of 16
  return note_launch(pdl_launch(tc_mlp_pair_kernel<STAGES>, dim3(2 * pairs), dim3(kTcThreads), L::TOTAL, s, map_a,
                                w1.map_hi[1][tc_bn_index(128)], w1.map_lo[1][tc_bn_index(128)],
                                w2.map_hi[1][tc_bn_index(64)], w2.map_lo[1][tc_bn_index(64)], map_y, p1, p2,
                                team));
}

}  // namespace ftb
