// CUDA runtime behind the C ABI: device weight replicas, per-thread execution
// contexts (one cudaMalloc'd block holding the planned arena and the staging
// buffers), CUDA-graph replay of the launch list, the host<->device copy
// pipeline and the kernel dispatch.
//
// Lifetime mirrors the reference's generated runtime (src/codegen.cpp:113-275):
// a context is leased per call from a pool owned by the calling thread, a
// nested call on the same thread leases another one, and after the first call
// on a thread no further allocation happens.  The allocation counters report
// the same events the reference counts (payload allocations and pool
// insertions, per thread; a process-wide total).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <string>
#include <unordered_map>
#include <vector>

#include "elementwise.cuh"
#include "engine.hpp"
#include "forgetune_b200.h"
#include "philox.cuh"
#include "simt_gemm.cuh"
#include "splitk_gemv.cuh"
#include "tc_pair_gemm.cuh"
#include "tc_mlp_pair.cuh"
#include "chain_gemv.cuh"
#include "tc_conv.cuh"
#include "narrow_gemm.cuh"

#define FTB_API extern "C" __attribute__((visibility("default")))

namespace ftb {

// ---------------------------------------------------------------------------
// status codes (include/forgetune_b200.h)
// ---------------------------------------------------------------------------
enum Status : int {
  ST_OK = 0,
  ST_NULL = -1,
  ST_INPUT = -2,
  ST_OUTPUT = -3,
  ST_ALLOC = -4,
  ST_DEVICE = -5,
  ST_CONFIG = -6,
};

static thread_local std::string t_last_error;

static void set_error(const std::string& s) { t_last_error = s; }

#define CUDA_TRY(expr)                                                                 \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess) {                                                           \
      set_error(std::string(#expr) + ": " + cudaGetErrorString(_e));                  \
      return ST_DEVICE;                                                                \
    }                                                                                  \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// ---------------------------------------------------------------------------
// device replica of the weights + launch list
// ---------------------------------------------------------------------------
struct Replica {
  int device = -1;
  float* weights = nullptr;  // blob weights followed by derived layouts
  size_t weight_floats = 0;
  std::vector<Step> steps;
  std::vector<ConvGeom> conv;  // per step (valid for ST_CONV)
  std::vector<TcWeights> tc;   // per step (valid when the tensor-core path may run)
  int sm_count = 148;
  // small-batch chain kernel: grid (0 = the launch list is not a chain of
  // dense layers it can run) and the widest layer input
  int chain_grid = 0;
  int64_t chain_kmax = 0;
  // error word the tensor-core kernel writes when a bounded wait gives up;
  // mapped pinned host memory, so the host reads it without a copy
  int* err_host = nullptr;
  int* err_dev = nullptr;
};

struct ExecCtx {
  int device = -1;
  cudaStream_t stream = nullptr;   // compute
  cudaStream_t h2d = nullptr;      // host -> device copies
  cudaStream_t d2h = nullptr;      // device -> host copies
  char* block = nullptr;           // the one allocation: arena | input | output
  size_t block_bytes = 0;
  char* arena = nullptr;
  float* d_in = nullptr;
  float* d_out = nullptr;
  std::vector<cudaEvent_t> ev_in, ev_out;  // per pipeline chunk
  cudaEvent_t ev_a = nullptr, ev_b = nullptr;
  std::vector<cudaEvent_t> prof;  // [slot][step + 1] step-boundary events
  // split-K workspace inside the block: partial sums and per-column-block tickets
  float* ws_part = nullptr;
  unsigned* ws_tickets = nullptr;
  // split-K partial sums of the SM-pair tensor-core GEMM
  float* ws_ksplit = nullptr;
  size_t ws_ksplit_floats = 0;
  // grid-barrier counters of the chain kernel and the two-layer kernel's
  // team counters (zero between launches)
  unsigned long long* chain_bar = nullptr;
  // the chain kernel's tagged hand-over words (kChainTagRows rows x the sum of the
  // layers' widths), or null when the launch list is not a chain of GEMMs
  unsigned long long* chain_tags = nullptr;
  size_t chain_tag_words = 0;
  unsigned* team_flags = nullptr;
  bool in_use = false;
  // pinned host staging for small host-to-host runs (allocated on first use):
  // the copies then run inside the forward's CUDA graph
  float* h_in = nullptr;
  float* h_out = nullptr;
  float* h_in_dev = nullptr;  // device addresses of the mapped staging buffers
  float* h_out_dev = nullptr;
  // completion word of a small chain run (mapped): the kernel's last CTA
  // sets it after its output is visible to the host
  volatile unsigned* h_done = nullptr;
  unsigned* h_done_dev = nullptr;
  struct CachedGraph {
    int64_t batch;
    const float* in;
    float* out;
    cudaGraphExec_t exec;
    bool staged;  // copies h_in -> in before and out -> h_out after the forward
  };
  std::vector<CachedGraph> graphs;
};

struct ThreadPool {
  std::vector<ExecCtx*> ctxs;
  size_t payload_allocs = 0;
  size_t block_insertions = 0;
};

struct Model;

// Registry of live models; leaked on purpose so thread-exit destructors that
// run during process teardown can still consult it safely.
struct Registry {
  std::mutex mu;
  std::unordered_map<uint64_t, Model*> live;
  std::atomic<uint64_t> next_uid{1};
};
static Registry* registry() {
  static Registry* r = new Registry;
  return r;
}

struct Model {
  uint64_t uid = 0;
  Program prog;
  std::vector<int> devices;  // empty: the caller's current device at first use
  std::vector<std::unique_ptr<Replica>> replicas;
  std::vector<ExecCtx*> all_ctxs;
  std::mutex mu;
  std::atomic<size_t> process_allocs{0};
  std::atomic<size_t> graph_kernels{0};  // kernel nodes of the most recently captured launch-list graph
  bool allow_tc = true;
  std::atomic<int> tc_stall_test{0};  // failure-detection hook, see ftb_model_set_fault_injection
};

static void destroy_ctx(ExecCtx* c) {
  if (!c) return;
  DeviceGuard g(c->device);
  for (auto& cg : c->graphs) cudaGraphExecDestroy(cg.exec);
  for (auto e : c->ev_in) cudaEventDestroy(e);
  for (auto e : c->ev_out) cudaEventDestroy(e);
  for (auto e : c->prof) cudaEventDestroy(e);
  if (c->ev_a) cudaEventDestroy(c->ev_a);
  if (c->ev_b) cudaEventDestroy(c->ev_b);
  if (c->stream) cudaStreamDestroy(c->stream);
  if (c->h2d) cudaStreamDestroy(c->h2d);
  if (c->d2h) cudaStreamDestroy(c->d2h);
  if (c->block) cudaFree(c->block);
  if (c->h_in) cudaFreeHost(c->h_in);
  if (c->h_out) cudaFreeHost(c->h_out);
  if (c->h_done) cudaFreeHost(const_cast<unsigned*>(c->h_done));
  delete c;
}

// thread-local pools keyed by (model uid, device)
struct PoolKey {
  uint64_t uid;
  int device;
  bool operator==(const PoolKey& o) const { return uid == o.uid && device == o.device; }
};
struct PoolKeyHash {
  size_t operator()(const PoolKey& k) const { return std::hash<uint64_t>()(k.uid * 131 + (uint64_t)k.device); }
};

struct ThreadPools {
  std::unordered_map<PoolKey, ThreadPool, PoolKeyHash> pools;
  ~ThreadPools() {
    // return this thread's contexts: free them if their model is still alive
    Registry* r = registry();
    std::lock_guard<std::mutex> lk(r->mu);
    for (auto& kv : pools) {
      auto it = r->live.find(kv.first.uid);
      if (it == r->live.end()) continue;
      Model* m = it->second;
      std::lock_guard<std::mutex> mlk(m->mu);
      for (ExecCtx* c : kv.second.ctxs) {
        auto pos = std::find(m->all_ctxs.begin(), m->all_ctxs.end(), c);
        if (pos != m->all_ctxs.end()) {
          m->all_ctxs.erase(pos);
          destroy_ctx(c);
        }
      }
    }
  }
};
static thread_local ThreadPools t_pools;

static ThreadPool& pool_of(Model* m, int dev) { return t_pools.pools[PoolKey{m->uid, dev}]; }

// A convolution the tensor-core path (tc_conv.cuh) runs: N = Cout >= 32
// output channels and an epilogue of a per-channel bias and ReLUs.
static bool conv_tc_candidate(const Step& s) {
  return s.kind == ST_CONV && s.N >= 32 && !(s.epi & (EPI_RESIDUAL | EPI_BIAS_ROWS)) &&
         tc_gemm_supported(tc_padded_k(s.K), s.N);
}

// Split-K partial sums per context (see launch_tc_pair_bn): 74 pairs x 256
// rows x 256 columns of fp32 covers every split it chooses on a B200.
static constexpr size_t kKsplitWorkspaceFloats = (size_t)74 * 256 * 256;

// ---------------------------------------------------------------------------
// replica creation: upload weights and derived layouts
// ---------------------------------------------------------------------------
static int make_replica(Model* m, int dev, Replica** out) {
  for (auto& r : m->replicas)
    if (r->device == dev) {
      *out = r.get();
      return ST_OK;
    }
  DeviceGuard guard(dev);
  auto rep = std::make_unique<Replica>();
  rep->device = dev;
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
  rep->sm_count = prop.multiProcessorCount;
  if (prop.major != 10) {
    set_error("forgetune_b200 kernels are built for sm_100a (B200); device " + std::to_string(dev) + " is sm_" +
              std::to_string(prop.major) + std::to_string(prop.minor));
    return ST_DEVICE;
  }
  const Graph& g = m->prog.graph;
  std::vector<float> host(g.weights);
  auto append = [&](size_t floats, size_t align_floats) {
    size_t off = (host.size() + align_floats - 1) / align_floats * align_floats;
    host.resize(off + floats, 0.0f);
    return off;
  };
  rep->steps = m->prog.steps;
  rep->conv.resize(rep->steps.size());
  rep->tc.resize(rep->steps.size());
  std::vector<uint64_t> ktab_off(rep->steps.size(), 0);
  for (size_t i = 0; i < rep->steps.size(); ++i) {
    Step& s = rep->steps[i];
    if (s.kind == ST_GEMM) {
      s.w_kn = s.b.offset;
      if (m->allow_tc && tc_gemm_supported(s.K, s.N)) {
        // W[K,N] -> W^T [N, Kp] as tf32 hi and lo parts
        const int64_t Kp = tc_padded_k(s.K);
        s.Kp = Kp;
        const size_t hi = append((size_t)s.N * Kp, 64);
        const size_t lo = append((size_t)s.N * Kp, 64);
        const float* w = g.weights.data() + s.b.offset;
        for (int64_t k = 0; k < s.K; ++k)
          for (int64_t n = 0; n < s.N; ++n) {
            const float v = w[k * s.N + n];
            const float h = tf32_round_host(v);
            host[hi + n * Kp + k] = h;
            host[lo + n * Kp + k] = tf32_round_host(v - h);
          }
        s.w_nk_hi = hi;
        s.w_nk_lo = lo;
      }
    } else if (s.kind == ST_CONV) {
      // OIHW [Cout, K] -> B[K, Cout]
      const size_t off = append((size_t)s.K * s.N, 16);
      const float* w = g.weights.data() + s.b.offset;
      for (int64_t co = 0; co < s.N; ++co)
        for (int64_t k = 0; k < s.K; ++k) host[off + k * s.N + co] = w[co * s.K + k];
      s.w_kn = off;
      if (m->allow_tc && conv_tc_candidate(s)) {
        // OIHW is already W^T [Cout, K]: tf32 hi / lo rows padded to Kp
        const int64_t Kp = tc_padded_k(s.K);
        s.Kp = Kp;
        const size_t hi = append((size_t)s.N * Kp, 64);
        const size_t lo = append((size_t)s.N * Kp, 64);
        for (int64_t co = 0; co < s.N; ++co)
          for (int64_t k = 0; k < s.K; ++k) {
            const float v = w[co * s.K + k];
            const float h = tf32_round_host(v);
            host[hi + co * Kp + k] = h;
            host[lo + co * Kp + k] = tf32_round_host(v - h);
          }
        s.w_nk_hi = hi;
        s.w_nk_lo = lo;
      }
      // k -> (input offset, dh*kh, dw*kw)
      ktab_off[i] = append((size_t)s.K * 4, 16);
      int32_t* t = reinterpret_cast<int32_t*>(host.data() + ktab_off[i]);
      int64_t k = 0;
      for (int64_t ci = 0; ci < s.Cin; ++ci)
        for (int64_t kh = 0; kh < s.Kh; ++kh)
          for (int64_t kw = 0; kw < s.Kw; ++kw, ++k) {
            t[4 * k + 0] = (int32_t)(ci * s.H * s.W + kh * s.conv.dh * s.W + kw * s.conv.dw);
            t[4 * k + 1] = (int32_t)(kh * s.conv.dh);
            t[4 * k + 2] = (int32_t)(kw * s.conv.dw);
            t[4 * k + 3] = 0;
          }
    }
  }
  // The small-batch chain kernel runs launch lists made only of dense layers
  // on the batch rows, with K a multiple of 4 (float4 rows) and one input row
  // fitting its shared memory; it reads an fp32 W^T [N, K] copy.
  {
    bool ok = !rep->steps.empty() && rep->steps.size() <= (size_t)kChainMaxLayers;
    int64_t kmax = 0, nmax = 0;
    for (const Step& s : rep->steps) {
      if (!ok) break;
      ok = s.kind == ST_GEMM && !s.static_rows && s.K >= 4 && s.K % 4 == 0 && s.N >= 1 &&
           s.K * 4 <= kChainSmemBytes && s.K * s.N <= ((int64_t)1 << 26) && s.b.space == SP_WEIGHT;
      kmax = std::max(kmax, s.K);
      nmax = std::max(nmax, s.N);
    }
    if (ok) {
      for (Step& s : rep->steps) {
        const size_t off = append((size_t)s.N * s.K, 16);
        const float* w = g.weights.data() + s.b.offset;
        for (int64_t n = 0; n < s.N; ++n)
          for (int64_t k = 0; k < s.K; ++k) host[off + n * s.K + k] = w[k * s.N + n];
        s.w_nk_f32 = off;
      }
      rep->chain_kmax = kmax;
      rep->chain_grid = (int)std::min<int64_t>(rep->sm_count, (nmax + kChainWarps - 1) / kChainWarps);
    }
  }
  rep->weight_floats = host.size();
  CUDA_TRY(cudaMalloc(&rep->weights, std::max<size_t>(host.size(), 1) * sizeof(float)));
  CUDA_TRY(cudaMemcpy(rep->weights, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice));
  for (size_t i = 0; i < rep->steps.size(); ++i) {
    const Step& s = rep->steps[i];
    if (s.kind == ST_CONV) {
      ConvGeom c;
      c.Cin = (int)s.Cin; c.H = (int)s.H; c.W = (int)s.W; c.Cout = (int)s.Cout;
      c.Kh = (int)s.Kh; c.Kw = (int)s.Kw; c.Ho = (int)s.Ho; c.Wo = (int)s.Wo;
      c.sh = (int)s.conv.sh; c.sw = (int)s.conv.sw; c.ph = (int)s.conv.ph;
      c.pw = (int)s.conv.pw; c.dh = (int)s.conv.dh; c.dw = (int)s.conv.dw;
      c.ktab = reinterpret_cast<const int4*>(rep->weights + ktab_off[i]);
      rep->conv[i] = c;
    }
    if ((s.kind == ST_GEMM || s.kind == ST_CONV) && s.w_nk_hi) {
      rep->tc[i].hi = rep->weights + s.w_nk_hi;
      rep->tc[i].lo = rep->weights + s.w_nk_lo;
      rep->tc[i].Kp = s.Kp;
      if (!tc_prepare_weights(rep->tc[i], s.N)) rep->tc[i] = TcWeights{};  // SIMT for this layer
    }
  }
  CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&rep->err_host), sizeof(int), cudaHostAllocMapped));
  *rep->err_host = 0;
  CUDA_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&rep->err_dev), rep->err_host, 0));
  *out = rep.get();
  m->replicas.push_back(std::move(rep));
  return ST_OK;
}

// ---------------------------------------------------------------------------
// execution contexts
// ---------------------------------------------------------------------------
static constexpr int kMaxChunks = 64;

static int alloc_block(ExecCtx* c, size_t bytes) {
  if (c->block) {
    cudaFree(c->block);
    c->block = nullptr;
    c->block_bytes = 0;
  }
  cudaError_t e = cudaMalloc(&c->block, std::max<size_t>(bytes, 256));
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error(std::string("device arena allocation of ") + std::to_string(bytes) + " bytes failed: " +
              cudaGetErrorString(e));
    c->block = nullptr;
    return ST_ALLOC;
  }
  c->block_bytes = bytes;
  return ST_OK;
}

static size_t round256(size_t v) { return (v + 255) / 256 * 256; }

static int layout_block(Model* m, ExecCtx* c, size_t min_bytes, bool* did_alloc) {
  const Program& p = m->prog;
  const size_t arena = round256(p.plan.arena_bytes);
  const size_t in_b = round256((size_t)p.max_batch * p.in_static_elems * sizeof(float));
  const size_t out_rows = p.output_dynamic ? (size_t)p.max_batch : 1;
  const size_t out_b = round256(out_rows * p.out_static_elems * sizeof(float));
  // split-K workspace sized for the widest GEMM: up to 64 slices x 16 rows x N
  int64_t max_n = 0;
  for (const Step& st : p.steps)
    if (st.kind == ST_GEMM) max_n = std::max(max_n, st.N);
  const size_t part_b = round256((size_t)kSkMaxSlices * 16 * (size_t)max_n * sizeof(float));
  const size_t tick_b = round256((size_t)((max_n + kSkCols - 1) / kSkCols + 1) * sizeof(unsigned));
  // split-K partial sums: it runs only when at most half the SM pairs have a
  // whole 256-row tile, so at most 74 x 256 x 256 floats
  bool any_tc = false;
  if (m->allow_tc)
    for (const Step& st : p.steps)
      if ((st.kind == ST_GEMM && tc_gemm_supported(st.K, st.N)) || conv_tc_candidate(st)) any_tc = true;
  const size_t ks_floats = any_tc ? kKsplitWorkspaceFloats : 0;
  const size_t ks_b = round256(ks_floats * sizeof(float));
  const size_t bar_b = 16384;  // chain-kernel barrier counters at 0, two-layer team counters at 256
  // chain-kernel tag words: kChainTagRows rows of every layer's output
  size_t tag_words = 0;
  {
    bool chain = !p.steps.empty() && p.steps.size() <= (size_t)kChainMaxLayers;
    int64_t sum_n = 0;
    for (const Step& st : p.steps) {
      chain = chain && st.kind == ST_GEMM;
      sum_n += st.N;
    }
    if (chain) tag_words = (size_t)kChainTagRows * (size_t)sum_n;
  }
  const size_t tag_b = round256(tag_words * sizeof(unsigned long long));
  const size_t need = std::max(arena + in_b + out_b + part_b + tick_b + ks_b + bar_b + tag_b, min_bytes);
  bool fresh = false;
  if (!c->block || c->block_bytes < need) {
    int rc = alloc_block(c, need);
    if (rc) return rc;
    if (did_alloc) *did_alloc = true;
    fresh = true;
    for (auto& cg : c->graphs) cudaGraphExecDestroy(cg.exec);
    c->graphs.clear();
  }
  c->arena = c->block;
  c->d_in = reinterpret_cast<float*>(c->block + arena);
  c->d_out = reinterpret_cast<float*>(c->block + arena + in_b);
  c->ws_part = max_n ? reinterpret_cast<float*>(c->block + arena + in_b + out_b) : nullptr;
  c->ws_tickets = max_n ? reinterpret_cast<unsigned*>(c->block + arena + in_b + out_b + part_b) : nullptr;
  c->ws_ksplit_floats = ks_floats;
  c->ws_ksplit = ks_floats ? reinterpret_cast<float*>(c->block + arena + in_b + out_b + part_b + tick_b) : nullptr;
  c->chain_bar = reinterpret_cast<unsigned long long*>(c->block + arena + in_b + out_b + part_b + tick_b + ks_b);
  c->team_flags = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(c->chain_bar) + 256);
  c->chain_tag_words = tag_words;
  c->chain_tags = tag_words ? reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(c->chain_bar) + bar_b)
                            : nullptr;
  static_assert(256 + kTcMlpTeamFlagWords * sizeof(unsigned) <= 16384, "team counters fit the counter area");
  if (fresh && c->ws_tickets) {
    // tickets start at zero; every split-K launch leaves them at zero
    if (cudaMemset(c->ws_tickets, 0, tick_b) != cudaSuccess) {
      cudaGetLastError();
      set_error("workspace initialisation failed");
      return ST_DEVICE;
    }
  }
  if (fresh) {
    // the chain kernel's counters start at zero (every launch leaves them at
    // zero; its launch counter only grows) and so do its tag words (tag 0
    // is never a launch's)
    if (cudaMemset(c->chain_bar, 0, bar_b + tag_b) != cudaSuccess) {
      cudaGetLastError();
      set_error("workspace initialisation failed");
      return ST_DEVICE;
    }
  }
  return ST_OK;
}

// Leases a free context of this thread on `dev`, creating one if all are busy.
static int lease(Model* m, int dev, ExecCtx** out) {
  ThreadPool& tp = pool_of(m, dev);
  for (ExecCtx* c : tp.ctxs)
    if (!c->in_use) {
      c->in_use = true;
      *out = c;
      return ST_OK;
    }
  DeviceGuard guard(dev);
  auto* c = new ExecCtx;
  c->device = dev;
  tp.block_insertions++;
  m->process_allocs++;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&c->h2d, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&c->d2h, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ev_a, cudaEventDefault) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ev_b, cudaEventDefault) != cudaSuccess) {
    cudaGetLastError();
    set_error("stream / event creation failed");
    destroy_ctx(c);
    return ST_DEVICE;
  }
  c->ev_in.resize(kMaxChunks);
  c->ev_out.resize(kMaxChunks);
  for (int i = 0; i < kMaxChunks; ++i) {
    if (cudaEventCreateWithFlags(&c->ev_in[i], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_out[i], cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      set_error("event creation failed");
      destroy_ctx(c);
      return ST_DEVICE;
    }
  }
  bool did = false;
  int rc = layout_block(m, c, 0, &did);
  if (rc) {
    destroy_ctx(c);
    return rc;
  }
  if (did) {
    tp.payload_allocs++;
    m->process_allocs++;
  }
  {
    std::lock_guard<std::mutex> lk(m->mu);
    m->all_ctxs.push_back(c);
  }
  tp.ctxs.push_back(c);
  c->in_use = true;
  *out = c;
  return ST_OK;
}

struct LeaseGuard {
  ExecCtx* c;
  ~LeaseGuard() {
    if (c) c->in_use = false;
  }
};

// ---------------------------------------------------------------------------
// kernel dispatch
// ---------------------------------------------------------------------------
template <int BM, int BN, int BK, int TM, int TN, bool EXACT, bool CONV>
static void launch_simt(const GemmArgs& a, cudaStream_t s) {
  constexpr int NT = (BM / TM) * (BN / TN);
  dim3 grid((unsigned)((a.M + BM - 1) / BM), (unsigned)((a.N + BN - 1) / BN));
  simt_gemm_kernel<BM, BN, BK, TM, TN, EXACT, CONV><<<grid, NT, 0, s>>>(a);
}

template <bool EXACT, bool CONV>
static void dispatch_simt(const GemmArgs& a, int sm_count, cudaStream_t s) {
  const int64_t M = a.M, N = a.N;
  if (M <= 16) {
    launch_simt<8, 32, 8, 1, 1, EXACT, CONV>(a, s);
  } else if (N <= 16) {
    launch_simt<64, 16, 8, 4, 1, EXACT, CONV>(a, s);
  } else if (((M + 127) / 128) * ((N + 127) / 128) >= 2 * sm_count) {
    launch_simt<128, 128, 8, 8, 8, EXACT, CONV>(a, s);
  } else {
    launch_simt<64, 64, 8, 4, 4, EXACT, CONV>(a, s);
  }
}

static int ew_grid(int64_t n, int sm_count) {
  int64_t b = (n + 255) / 256;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, (int64_t)sm_count * 8));
}

static void copy_floats(const float* a, float* y, int64_t n, int sm, cudaStream_t s) {
  if (n <= 0) return;
  if (((uintptr_t)a % 16 == 0) && ((uintptr_t)y % 16 == 0) && n % 4 == 0) {
    copy4_kernel<<<ew_grid(n / 4, sm), 256, 0, s>>>(reinterpret_cast<const float4*>(a), reinterpret_cast<float4*>(y),
                                                  n / 4);
  } else {
    ew_unary_kernel<EW_COPY><<<ew_grid(n, sm), 256, 0, s>>>(a, y, n);
  }
}

// Enqueues the launch list for `batch` rows on stream s.  With `marks`
// (steps + 1 events) an event is recorded before every step and after the
// last one, so per-step device times can be read back afterwards.
// Whether the launch list at this batch runs as the one-launch chain kernel
// (every condition of enqueue's chain branch that does not depend on the
// buffers' addresses).
static bool chain_takes(const Model* m, const Replica* rep, int64_t batch) {
  const int policy = m->prog.graph.kernel_policy;
  if (!(policy == KP_AUTO || policy == KP_SIMT) || rep->chain_grid <= 0 || batch < 1 || batch > kChainMaxRows ||
      (size_t)batch * (size_t)rep->chain_kmax * 4 > (size_t)kChainSmemBytes)
    return false;
  for (const Step& st : rep->steps) {
    const TuneRecord* tr = st.tuned_for(batch);
    if (tr && tr->family != TF_HEURISTIC) return false;
  }
  return true;
}

static int enqueue(const Model* m, const Replica* rep, ExecCtx* c, const float* in, float* out, int64_t batch,
                   cudaStream_t s, cudaEvent_t* marks = nullptr) {
  char* arena = c->arena;
  const int policy = m->prog.graph.kernel_policy;
  const bool exact = policy == KP_SIMT_EXACT;
  auto ptr = [&](const Operand& o) -> float* {
    switch (o.space) {
      case SP_INPUT: return const_cast<float*>(in);
      case SP_OUTPUT: return out;
      case SP_ARENA: return reinterpret_cast<float*>(arena + o.offset);
      case SP_WEIGHT: return rep->weights + o.offset;
      default: return nullptr;
    }
  };
  const int sm = rep->sm_count;
  // Small batches of a chain of dense layers: the whole forward pass in one
  // launch (chain_gemv.cuh), unless a tuned entry picks kernels for this batch.
  if (!exact && (policy == KP_AUTO || policy == KP_SIMT) && rep->chain_grid > 0 && c->chain_bar && batch >= 1 &&
      batch <= kChainMaxRows && (size_t)batch * (size_t)rep->chain_kmax * 4 <= (size_t)kChainSmemBytes) {
    bool take = true;
    ChainParams p;
    std::memset(&p, 0, sizeof(p));
    p.n_layers = (int)rep->steps.size();
    p.M = (int)batch;
    p.bar = c->chain_bar;
    p.err = rep->err_dev;
    p.done = (in == c->h_in_dev && c->h_done_dev) ? c->h_done_dev : nullptr;
    p.stall_test = m->tc_stall_test.load();
    // tagged hand-over: the layers whose outputs a later layer reads
    size_t tag_next = 0;
    bool tags_ok = c->chain_tags != nullptr;
    for (size_t i = 0; i < rep->steps.size() && take; ++i) {
      const Step& st = rep->steps[i];
      const TuneRecord* tr = st.tuned_for(batch);
      if (tr && tr->family != TF_HEURISTIC) take = false;
      ChainLayer& L = p.layer[i];
      L.a = ptr(st.a);
      L.w = rep->weights + st.w_nk_f32;
      L.bias = (st.bias.space && (st.epi & (EPI_BIAS_FIRST | EPI_BIAS_LAST))) ? ptr(st.bias) : nullptr;
      L.res = st.res.space ? ptr(st.res) : nullptr;
      L.y = ptr(st.out);
      L.K = (int)st.K;
      L.N = (int)st.N;
      L.epi = st.epi;
      if (reinterpret_cast<uintptr_t>(L.a) & 15u) take = false;  // float4 rows
      L.tag_off = -1;
      L.a_src = -1;
      L.res_src = -1;
      for (size_t j = 0; j < i; ++j) {
        const float* out_j = ptr(rep->steps[j].out);
        if (out_j == L.a) L.a_src = (int)j;
        if (L.res && out_j == L.res) L.res_src = (int)j;
      }
      for (int src : {L.a_src, L.res_src}) {
        if (src >= 0 && p.layer[src].tag_off < 0) {
          p.layer[src].tag_off = (int)tag_next;
          tag_next += (size_t)batch * (size_t)rep->steps[(size_t)src].N;
        }
      }
    }
    if (tags_ok && batch <= kChainTagRows && tag_next <= c->chain_tag_words) p.tags = c->chain_tags;
    const size_t smem = take ? chain_plan(p, rep->chain_grid) : 0;
    if (take && smem > 0) {
      if (marks) cudaEventRecord(marks[0], s);
      if (launch_chain(p, rep->chain_grid, smem, s) != 0) {
        set_error(std::string("chain kernel launch failed: ") + cudaGetErrorString(take_launch_error()));
        return ST_DEVICE;
      }
      if (marks)
        for (size_t i = 1; i <= rep->steps.size(); ++i) cudaEventRecord(marks[i], s);
      return ST_OK;
    }
  }
  // steps already computed by an earlier launch: a head fused into the
  // previous GEMM's epilogue, the second layer of a two-layer kernel and its head
  size_t skip_step = (size_t)-1, skip_step2 = (size_t)-1;
  for (size_t i = 0; i < rep->steps.size(); ++i) {
    const Step& st = rep->steps[i];
    const int64_t rows = st.static_rows ? 1 : batch;
    if (marks) cudaEventRecord(marks[i], s);
    if (i == skip_step || i == skip_step2) continue;
    switch (st.kind) {
      case ST_GEMM:
      case ST_CONV: {
        GemmArgs a{};
        a.A = ptr(st.a);
        a.B = st.kind == ST_CONV ? rep->weights + st.w_kn : ptr(st.b);
        a.bias = st.bias.space ? ptr(st.bias) : nullptr;
        a.res = st.res.space ? ptr(st.res) : nullptr;
        a.Y = ptr(st.out);
        a.N = (int)st.N;
        a.K = (int)st.K;
        a.epi = st.epi;
        const int64_t M = st.kind == ST_CONV ? (st.static_rows ? st.rows_per_sample : batch) * st.Ho * st.Wo
                                             : (st.static_rows ? st.rows_per_sample : batch);
        a.M = (int)M;
        if (st.kind == ST_CONV) {
          a.conv = rep->conv[i];
          const TcWeights& tw = rep->tc[i];
          int tc_rc = 1;  // 1: not taken
          // convolutions of 32 output channels too: their implicit GEMMs
          // have many rows, and the SIMT convolution is what they replace
          if (!exact && tw.maps_ready && M <= 0x7fffffff &&
              (policy == KP_TCGEN05 || (policy == KP_AUTO && M >= 128 && st.N >= 32 && st.Kp >= 32))) {
            TcConvParams cp;
            std::memset(&cp, 0, sizeof(cp));
            cp.x = a.A;
            cp.ktab = a.conv.ktab;
            cp.bias = a.bias;
            cp.res = a.res;
            cp.y = a.Y;
            cp.M = (int)M;
            cp.N = (int)st.N;
            cp.K = (int)st.K;
            cp.Cin = (int)st.Cin;
            cp.H = (int)st.H;
            cp.W = (int)st.W;
            cp.Ho = (int)st.Ho;
            cp.Wo = (int)st.Wo;
            cp.sh = (int)st.conv.sh;
            cp.sw = (int)st.conv.sw;
            cp.ph = (int)st.conv.ph;
            cp.pw = (int)st.conv.pw;
            cp.epi = st.epi;
            cp.err = rep->err_dev;
            cp.stall_test = m->tc_stall_test.load();
            tc_rc = launch_tc_conv(cp, tw, sm, s);
            if (tc_rc < 0) {
              set_error(std::string("tensor-core convolution launch failed: ") +
                        cudaGetErrorString(take_launch_error()));
              return ST_DEVICE;
            }
          }
          if (tc_rc == 0) {
            // implicit GEMM on the tensor cores, NCHW stores from the epilogue
          } else if (exact) {
            dispatch_simt<true, true>(a, sm, s);
          } else {
            dispatch_simt<false, true>(a, sm, s);
          }
        } else {
          const TcWeights& tw = rep->tc[i];
          // a tuned entry for this batch overrides the shape rules (never in
          // the bit-exact policy); an entry whose family cannot run this shape
          // falls back to them
          const TuneRecord* tr = exact ? nullptr : st.tuned_for(batch);
          const int fam = tr ? tr->family : TF_HEURISTIC;
          const bool want_splitk = fam == TF_SPLITK || (fam == TF_HEURISTIC && policy != KP_TCGEN05);
          if (!exact && M <= 16 && c->ws_part && want_splitk && fam != TF_SIMT && fam != TF_TCGEN05) {
            SplitKArgs sk{};
            sk.A = a.A;
            sk.B = a.B;
            sk.bias = a.bias;
            sk.res = a.res;
            sk.Y = a.Y;
            sk.part = c->ws_part;
            sk.tickets = c->ws_tickets;
            sk.M = (int)M;
            sk.N = (int)st.N;
            sk.K = (int)st.K;
            sk.epi = st.epi;
            cudaError_t lerr = cudaSuccess;
            const int rc = launch_splitk(sk, sm, s, &lerr);
            if (rc < 0) {
              set_error(std::string("split-K GEMM launch failed: ") + cudaGetErrorString(lerr));
              return ST_DEVICE;
            }
            if (rc == 0) break;
          }
          // this layer and the next in one kernel: by shape when neither step
          // carries a tile configuration or a tuned entry, or when asked for
          // (pair 4)
          if (st.mlp_step >= 0 && !exact && (policy == KP_AUTO || policy == KP_TCGEN05)) {
            const Step& s2 = rep->steps[(size_t)st.mlp_step];
            const TcWeights& tw2 = rep->tc[(size_t)st.mlp_step];
            auto plain = [](const Step& x) { return x.tc_bn == 0 && x.tc_bk == 0 && x.tc_mh == 0 && x.tc_pair == 0; };
            const TuneRecord* tr2 = s2.tuned_for(batch);
            const int asked_pair = tr ? tr->pair : st.tc_pair;
            const bool asked = asked_pair == 4 || asked_pair == 5;
            // few tiles: layer 1 split over teams of pairs (by shape, or pair 5)
            const bool team_ok = asked_pair == 5 || !asked;
            const bool by_shape = !tr && !tr2 && plain(st) && plain(s2) && tc_gemm_profitable(M, st.K, st.N) &&
                                  tc_gemm_profitable(M, s2.K, s2.N);
            if (asked || by_shape) {
              TcArgs t1{}, t2{};
              t1.A = a.A;
              t1.bias = a.bias;
              t1.M = M;
              t1.N = st.N;
              t1.K = st.K;
              t1.Kp = tw.Kp;
              t1.epi = st.epi;
              t1.stall_test = m->tc_stall_test.load();
              t1.ws = c->ws_ksplit;
              t1.ws_floats = c->ws_ksplit_floats;
              t2.A = nullptr;
              t2.bias = s2.bias.space ? ptr(s2.bias) : nullptr;
              t2.Y = ptr(s2.out);
              t2.M = M;
              t2.N = s2.N;
              t2.K = s2.K;
              t2.Kp = tw2.Kp;
              t2.epi = s2.epi;
              const bool head = s2.head_step >= 0 && (tr2 ? tr2->fuse_head : s2.fuse_head);
              if (head) {
                const Step& hs = rep->steps[(size_t)s2.head_step];
                t2.head.w = ptr(hs.b);
                t2.head.bias = hs.bias.space ? ptr(hs.bias) : nullptr;
                t2.head.y = ptr(hs.out);
                t2.head.n = (int)hs.N;
                t2.head.epi = hs.epi;
              }
              const int mrc = launch_tc_mlp(t1, tw, t2, tw2, rep->err_dev, s, team_ok ? c->team_flags : nullptr);
              if (mrc < 0) {
                set_error(std::string("two-layer tensor-core launch failed: ") +
                          cudaGetErrorString(take_launch_error()));
                return ST_DEVICE;
              }
              if (mrc == 0) {
                skip_step = (size_t)st.mlp_step;
                if (head) skip_step2 = (size_t)s2.head_step;
                break;
              }
            }
          }
          const bool tc_ok = tw.maps_ready && !exact && fam != TF_SIMT && fam != TF_SPLITK &&
                             (fam == TF_TCGEN05 || policy == KP_TCGEN05 ||
                              (policy == KP_AUTO && tc_gemm_profitable(M, st.K, st.N)));
          int tc_rc = 1;  // 1: not taken
          if (tc_ok) {
            TcArgs t{};
            t.A = a.A;
            t.w_hi = tw.hi;
            t.w_lo = tw.lo;
            t.bias = a.bias;
            t.res = a.res;
            t.Y = a.Y;
            t.M = M;
            t.N = st.N;
            t.K = st.K;
            t.Kp = tw.Kp;
            t.epi = st.epi;
            t.stall_test = m->tc_stall_test.load();
            t.ws = c->ws_ksplit;
            t.ws_floats = c->ws_ksplit_floats;
            TcConfig cfg;
            cfg.bn = tr ? tr->bn : st.tc_bn;
            cfg.bk = tr ? tr->bk : st.tc_bk;
            cfg.mh = tr ? tr->mh : st.tc_mh;
            cfg.pair = tr ? tr->pair : st.tc_pair;
            if (cfg.pair >= 4) cfg.pair = 0;  // the two-layer kernel did not apply: by shape
            const bool fuse_head = tr ? tr->fuse_head : st.fuse_head;
            if (st.head_step >= 0 && fuse_head) {
              const Step& hs = rep->steps[(size_t)st.head_step];
              t.head.w = ptr(hs.b);
              t.head.bias = hs.bias.space ? ptr(hs.bias) : nullptr;
              t.head.y = ptr(hs.out);
              t.head.n = (int)hs.N;
              t.head.epi = hs.epi;
            }
            tc_rc = launch_tc_gemm(t, tw, rep->err_dev, sm, s, cfg);
            if (tc_rc == 1 && t.head.n > 0) {
              // the fused form does not apply: plain tensor-core GEMM, head runs as its own step
              t.head = TcHead{};
              tc_rc = launch_tc_gemm(t, tw, rep->err_dev, sm, s, cfg);
            } else if (tc_rc == 0 && t.head.n > 0) {
              skip_step = (size_t)st.head_step;
            }
            if (tc_rc < 0) {
              set_error(std::string("tensor-core GEMM launch failed: ") + cudaGetErrorString(take_launch_error()));
              return ST_DEVICE;
            }
          }
          // few output columns (small heads): the narrow-N kernel
          int nrc = 1;
          if (tc_rc != 0 && !exact && st.N <= kNarrowMaxN) {
            nrc = launch_narrow_gemm(a.A, a.B, a.bias, a.res, a.Y, M, st.K, st.N, a.epi, sm, s);
            if (nrc < 0) {
              set_error(std::string("narrow GEMM launch failed: ") + cudaGetErrorString(take_launch_error()));
              return ST_DEVICE;
            }
          }
          if (tc_rc == 0 || nrc == 0) {
            // launched on the tensor cores / the narrow-N kernel
          } else if (exact) {
            dispatch_simt<true, false>(a, sm, s);
          } else {
            dispatch_simt<false, false>(a, sm, s);
          }
        }
        break;
      }
      case ST_ADD_SAME:
      case ST_ADD_ROW:
      case ST_ADD_CHANNEL:
      case ST_MUL_SAME:
      case ST_MUL_ROW:
      case ST_MUL_CHANNEL: {
        const int64_t n = rows * st.elems_per_sample;
        if (n <= 0) break;
        const float* A = ptr(st.a);
        const float* B = ptr(st.b);
        float* Y = ptr(st.out);
        const int g = ew_grid(n, sm);
        switch (st.kind) {
          case ST_ADD_SAME: ew_binary_kernel<EW_ADD, BC_SAME><<<g, 256, 0, s>>>(A, B, Y, n, 1, 1); break;
          case ST_ADD_ROW: ew_binary_kernel<EW_ADD, BC_ROW><<<g, 256, 0, s>>>(A, B, Y, n, st.row_len, 1); break;
          case ST_ADD_CHANNEL:
            ew_binary_kernel<EW_ADD, BC_CHANNEL><<<g, 256, 0, s>>>(A, B, Y, n, st.row_len, st.channels);
            break;
          case ST_MUL_SAME: ew_binary_kernel<EW_MUL, BC_SAME><<<g, 256, 0, s>>>(A, B, Y, n, 1, 1); break;
          case ST_MUL_ROW: ew_binary_kernel<EW_MUL, BC_ROW><<<g, 256, 0, s>>>(A, B, Y, n, st.row_len, 1); break;
          default:
            ew_binary_kernel<EW_MUL, BC_CHANNEL><<<g, 256, 0, s>>>(A, B, Y, n, st.row_len, st.channels);
            break;
        }
        break;
      }
      case ST_RELU:
      case ST_SIGMOID:
      case ST_TANH: {
        const int64_t n = rows * st.elems_per_sample;
        if (n <= 0) break;
        const int g = ew_grid(n, sm);
        if (st.kind == ST_RELU)
          ew_unary_kernel<EW_RELU><<<g, 256, 0, s>>>(ptr(st.a), ptr(st.out), n);
        else if (st.kind == ST_SIGMOID)
          ew_unary_kernel<EW_SIGMOID><<<g, 256, 0, s>>>(ptr(st.a), ptr(st.out), n);
        else
          ew_unary_kernel<EW_TANH><<<g, 256, 0, s>>>(ptr(st.a), ptr(st.out), n);
        break;
      }
      case ST_COPY:
      case ST_FILL_CONST: {
        const float* A = ptr(st.a);
        float* Y = ptr(st.out);
        if (A != Y) copy_floats(A, Y, rows * st.elems_per_sample, sm, s);
        break;
      }
      default:
        set_error("internal: unknown step kind");
        return ST_DEVICE;
    }
  }
  if (marks) cudaEventRecord(marks[rep->steps.size()], s);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("kernel launch failed: ") + cudaGetErrorString(e));
    return ST_DEVICE;
  }
  return ST_OK;
}

// After a synchronising call: did a tensor-core kernel give up on a wait?
static int check_kernel_error(const Replica* rep) {
  const volatile int* e = rep->err_host;
  if (e && *e != 0) {
    set_error("kernel aborted: a bounded wait (tensor-core pipeline, grid barrier or hand-over) exceeded its limit (code " +
              std::to_string(*e) + ")");
    return ST_DEVICE;
  }
  return ST_OK;
}

static constexpr size_t kMaxGraphs = 16;

// Replays the launch list for (batch, in, out) as a cached CUDA graph.
// With `staged`, the graph also copies in_bytes from the context's pinned
// input staging to `in` first and out_bytes from `out` to the output staging
// last, so a small host-to-host run is one graph launch.
static int run_graph(Model* m, Replica* rep, ExecCtx* c, const float* in, float* out, int64_t batch,
                     cudaStream_t s, bool staged = false, size_t in_bytes = 0, size_t out_bytes = 0) {
  for (auto& g : c->graphs)
    if (g.batch == batch && g.in == in && g.out == out && g.staged == staged) {
      CUDA_TRY(cudaGraphLaunch(g.exec, s));
      return ST_OK;
    }
  cudaGraph_t graph = nullptr;
  CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  int rc = ST_OK;
  if (staged && cudaMemcpyAsync(const_cast<float*>(in), c->h_in, in_bytes, cudaMemcpyHostToDevice, c->stream) !=
                    cudaSuccess) {
    set_error("staged input copy could not be captured");
    rc = ST_DEVICE;
  }
  if (rc == ST_OK) rc = enqueue(m, rep, c, in, out, batch, c->stream);
  if (rc == ST_OK && staged &&
      cudaMemcpyAsync(c->h_out, out, out_bytes, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) {
    set_error("staged output copy could not be captured");
    rc = ST_DEVICE;
  }
  cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) {
    set_error(std::string("graph capture failed: ") + cudaGetErrorString(e));
    return ST_DEVICE;
  }
  {
    // kernels one replay launches (the step list minus fused-away steps,
    // plus the extra passes of split-K and convolutions)
    size_t n = 0, k = 0;
    cudaGraphGetNodes(graph, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    if (n && cudaGraphGetNodes(graph, nodes.data(), &n) == cudaSuccess)
      for (cudaGraphNode_t node : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(node, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++k;
      }
    m->graph_kernels.store(k);
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    set_error(std::string("graph instantiate failed: ") + cudaGetErrorString(e));
    return ST_DEVICE;
  }
  if (c->graphs.size() >= kMaxGraphs) {
    cudaGraphExecDestroy(c->graphs.front().exec);
    c->graphs.erase(c->graphs.begin());
  }
  c->graphs.push_back({batch, in, out, exec, staged});
  CUDA_TRY(cudaGraphLaunch(exec, s));
  return ST_OK;
}

static int resolve_devices(Model* m, std::vector<int>* devs) {
  if (!m->devices.empty()) {
    *devs = m->devices;
    return ST_OK;
  }
  int d = 0;
  CUDA_TRY(cudaGetDevice(&d));
  devs->assign(1, d);
  return ST_OK;
}

// host-to-host runs whose input and output each fit this many bytes go
// through pinned staging with the copies inside the graph
static constexpr size_t kHostStageBytes = 256u << 10;
// Every CTA of the chain kernel reads all input rows: read straight from
// mapped host memory only while that stays a few PCIe round trips (one
// row of the tiny MLP on 32 CTAs is 100 KB), else copy them in first.
static constexpr size_t kZeroCopyReadBytes = 128u << 10;

// rows per pipeline chunk so one chunk's input is about 32 MiB
static int64_t chunk_rows_for(const Program& p, int64_t batch) {
  const int64_t per_row = std::max<int64_t>(1, p.in_static_elems * 4);
  int64_t rows = std::max<int64_t>(4096, (32ll << 20) / per_row);
  rows = std::max<int64_t>(rows, (batch + kMaxChunks - 1) / kMaxChunks);
  return rows;
}

// Host buffers in, host buffers out, on one device: chunked pipeline
// H2D(c) || compute(c-1) || D2H(c-2) over three streams.
static int run_host_one(Model* m, int dev, const float* in, float* out, int64_t batch) {
  Replica* rep = nullptr;
  int rc;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    rc = make_replica(m, dev, &rep);
  }
  if (rc) return rc;
  ExecCtx* c = nullptr;
  rc = lease(m, dev, &c);
  if (rc) return rc;
  LeaseGuard lg{c};
  DeviceGuard guard(dev);
  const Program& p = m->prog;
  const bool chunked = p.dynamic && p.output_dynamic && batch > chunk_rows_for(p, batch);
  if (!chunked) {
    const size_t in_b = (size_t)(p.dynamic ? batch : 1) * p.in_static_elems * 4;
    const size_t out_b = (size_t)(p.output_dynamic ? batch : 1) * p.out_static_elems * 4;
    *rep->err_host = 0;  // the previous synchronous run on this replica has finished
    if (in_b <= kHostStageBytes && out_b <= kHostStageBytes) {
      // small run: host memcpy into pinned staging, one graph launch that
      // copies in, computes and copies out, one synchronisation
      if (!c->h_in) {
        if (cudaHostAlloc(reinterpret_cast<void**>(&c->h_in), kHostStageBytes, cudaHostAllocMapped) != cudaSuccess ||
            cudaHostAlloc(reinterpret_cast<void**>(&c->h_out), kHostStageBytes, cudaHostAllocMapped) != cudaSuccess ||
            cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->h_in_dev), c->h_in, 0) != cudaSuccess ||
            cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->h_out_dev), c->h_out, 0) != cudaSuccess) {
          cudaGetLastError();
          set_error("pinned host staging allocation failed");
          return ST_ALLOC;
        }
        unsigned* done = nullptr;
        if (cudaHostAlloc(reinterpret_cast<void**>(&done), 64, cudaHostAllocMapped) != cudaSuccess ||
            cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->h_done_dev), done, 0) != cudaSuccess) {
          cudaGetLastError();
          if (done) cudaFreeHost(done);
          c->h_done_dev = nullptr;  // completion by stream query only
        } else {
          c->h_done = done;
        }
      }
      std::memcpy(c->h_in, in, in_b);
      const bool zero_copy = chain_takes(m, rep, batch) && in_b * (size_t)rep->chain_grid <= kZeroCopyReadBytes;
      const bool by_word = zero_copy && c->h_done;
      if (by_word) {
        *c->h_done = 0u;  // the previous run's word was seen: no write of it is in flight
        std::atomic_thread_fence(std::memory_order_seq_cst);
      }
      if (zero_copy) {
        // the one-launch chain reads its input rows from and writes its
        // output to the mapped staging buffers itself: no copy at all
        rc = run_graph(m, rep, c, c->h_in_dev, c->h_out_dev, batch, c->stream);
      } else {
        rc = run_graph(m, rep, c, c->d_in, c->d_out, batch, c->stream, true, in_b, out_b);
      }
      if (rc) return rc;
      // a few microseconds of work: poll instead of sleeping in the driver --
      // the chain kernel's completion word where it has one (the output is
      // visible to the host once it is set), with the stream queried now and
      // then for errors; else the stream
      cudaError_t q = cudaSuccess;
      for (uint64_t it = 0;; ++it) {
        if (by_word && *c->h_done) break;
        if (!by_word || (it & 255u) == 255u) {
          q = cudaStreamQuery(c->stream);
          if (q != cudaErrorNotReady) break;
        }
      }
      std::atomic_thread_fence(std::memory_order_acquire);
      if (q != cudaSuccess && q != cudaErrorNotReady) {
        set_error(std::string("small run: ") + cudaGetErrorString(q));
        return ST_DEVICE;
      }
      rc = check_kernel_error(rep);
      if (rc) return rc;
      std::memcpy(out, c->h_out, out_b);
      return ST_OK;
    }
    CUDA_TRY(cudaMemcpyAsync(c->d_in, in, in_b, cudaMemcpyHostToDevice, c->stream));
    rc = run_graph(m, rep, c, c->d_in, c->d_out, batch, c->stream);
    if (rc) return rc;
    CUDA_TRY(cudaMemcpyAsync(out, c->d_out, out_b, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return check_kernel_error(rep);
  }
  *rep->err_host = 0;
  const int64_t cr = chunk_rows_for(p, batch);
  const int64_t nch = (batch + cr - 1) / cr;
  const int64_t fi = p.in_static_elems, fo = p.out_static_elems;
  for (int64_t k = 0; k < nch; ++k) {
    const int64_t r0 = k * cr, r1 = std::min(batch, r0 + cr);
    CUDA_TRY(cudaMemcpyAsync(c->d_in + r0 * fi, in + r0 * fi, (size_t)(r1 - r0) * fi * 4, cudaMemcpyHostToDevice,
                             c->h2d));
    CUDA_TRY(cudaEventRecord(c->ev_in[k], c->h2d));
  }
  for (int64_t k = 0; k < nch; ++k) {
    const int64_t r0 = k * cr, r1 = std::min(batch, r0 + cr);
    CUDA_TRY(cudaStreamWaitEvent(c->stream, c->ev_in[k], 0));
    // chunks are thousands of rows: launch directly, no graph per chunk address
    rc = enqueue(m, rep, c, c->d_in + r0 * fi, c->d_out + r0 * fo, r1 - r0, c->stream);
    if (rc) return rc;
    CUDA_TRY(cudaEventRecord(c->ev_out[k], c->stream));
    CUDA_TRY(cudaStreamWaitEvent(c->d2h, c->ev_out[k], 0));
    CUDA_TRY(cudaMemcpyAsync(out + r0 * fo, c->d_out + r0 * fo, (size_t)(r1 - r0) * fo * 4,
                             cudaMemcpyDeviceToHost, c->d2h));
  }
  CUDA_TRY(cudaStreamSynchronize(c->d2h));
  CUDA_TRY(cudaStreamSynchronize(c->stream));
  return check_kernel_error(rep);
}

static int run_host(Model* m, const float* in, float* out, int64_t batch) {
  std::vector<int> devs;
  int rc = resolve_devices(m, &devs);
  if (rc) return rc;
  const Program& p = m->prog;
  if (devs.size() == 1 || !p.dynamic || !p.output_dynamic || batch < (int64_t)devs.size()) {
    return run_host_one(m, devs[0], in, out, batch);
  }
  // contiguous row blocks, one per device; the host thread drives them in turn
  const int64_t G = (int64_t)devs.size();
  const int64_t per = (batch + G - 1) / G;
  std::vector<std::thread> workers;
  std::vector<int> rcs(devs.size(), 0);
  std::vector<std::string> errs(devs.size());
  for (int64_t g = 0; g < G; ++g) {
    const int64_t r0 = g * per, r1 = std::min(batch, r0 + per);
    if (r1 <= r0) continue;
    workers.emplace_back([&, g, r0, r1]() {
      rcs[g] = run_host_one(m, devs[g], in + r0 * p.in_static_elems, out + r0 * p.out_static_elems, r1 - r0);
      if (rcs[g]) errs[g] = t_last_error;
    });
  }
  for (auto& w : workers) w.join();
  for (size_t g = 0; g < rcs.size(); ++g)
    if (rcs[g]) {
      set_error("device " + std::to_string(devs[g]) + ": " + errs[g]);
      return rcs[g];
    }
  return ST_OK;
}

// Reference validation for the three run entry points (src/codegen.cpp:722-1040).
// api: 0 = forgetune_run, 1 = forgetune_run_v1, 2 = forgetune_run_v2.
static int validate(const Program& p, const float* in, size_t in_count, const float* out, size_t out_count,
                    int64_t* batch, int api) {
  if (p.dynamic) {
    if (api == 2 && *batch <= 0) return ST_INPUT;
    if (api == 1) *batch = -1;
    if (!in || !out) return ST_NULL;
    const int64_t si = p.in_static_elems;
    if (*batch <= 0) {
      if (si == 0 || in_count == 0 || in_count % (size_t)si != 0) return ST_INPUT;
      *batch = (int64_t)(in_count / (size_t)si);
    }
    if (*batch <= 0 || *batch > p.max_batch) return ST_INPUT;
    if (in_count != (size_t)(*batch * si)) return ST_INPUT;
    const size_t want_out = p.output_dynamic ? (size_t)(*batch * p.out_static_elems) : (size_t)p.out_static_elems;
    if (out_count != want_out) return ST_OUTPUT;
    return ST_OK;
  }
  if (api == 2 && (*batch <= 0 || *batch != p.static_batch)) return ST_INPUT;
  if (!in || !out) return ST_NULL;
  if (in_count != (size_t)p.in_static_elems) return ST_INPUT;
  if (out_count != (size_t)p.out_static_elems) return ST_OUTPUT;
  *batch = p.static_batch;
  return ST_OK;
}

}  // namespace ftb

using namespace ftb;

// ===========================================================================
// C ABI
// ===========================================================================
FTB_API const char* ftb_last_error(void) { return t_last_error.c_str(); }

FTB_API int ftb_describe_blob(const void* blob, size_t bytes, char* buf, size_t cap) {
  try {
    Program p = build_program(blob, bytes);
    std::string s = p.describe();
    if (buf && cap) {
      size_t n = std::min(cap - 1, s.size());
      std::memcpy(buf, s.data(), n);
      buf[n] = 0;
    }
    return (int)s.size();
  } catch (const std::exception& e) {
    set_error(e.what());
    return ST_CONFIG;
  }
}

FTB_API int ftb_model_create(const void* blob, size_t bytes, void** out_model) {
  if (!blob || !out_model) return ST_NULL;
  try {
    auto* m = new Model;
    m->prog = build_program(blob, bytes);
    Registry* r = registry();
    m->uid = r->next_uid++;
    {
      std::lock_guard<std::mutex> lk(r->mu);
      r->live[m->uid] = m;
    }
    *out_model = m;
    return ST_OK;
  } catch (const std::exception& e) {
    set_error(e.what());
    return ST_CONFIG;
  }
}

FTB_API void ftb_model_destroy(void* handle) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return;
  Registry* r = registry();
  {
    std::lock_guard<std::mutex> lk(r->mu);
    r->live.erase(m->uid);
  }
  for (ExecCtx* c : m->all_ctxs) destroy_ctx(c);
  m->all_ctxs.clear();
  for (auto& rep : m->replicas) {
    DeviceGuard g(rep->device);
    if (rep->weights) cudaFree(rep->weights);
    if (rep->err_host) cudaFreeHost(rep->err_host);
  }
  m->replicas.clear();
  delete m;
}

FTB_API int ftb_model_set_devices(void* handle, const int* ids, int n) {
  auto* m = static_cast<Model*>(handle);
  if (!m || (n > 0 && !ids)) return ST_NULL;
  int count = 0;
  CUDA_TRY(cudaGetDeviceCount(&count));
  std::vector<int> d;
  for (int i = 0; i < n; ++i) {
    if (ids[i] < 0 || ids[i] >= count) {
      set_error("device id " + std::to_string(ids[i]) + " out of range");
      return ST_CONFIG;
    }
    d.push_back(ids[i]);
  }
  std::lock_guard<std::mutex> lk(m->mu);
  m->devices = d;
  return ST_OK;
}

FTB_API int ftb_model_set_policy(void* handle, int policy) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return ST_NULL;
  if (policy < KP_AUTO || policy > KP_TCGEN05) return ST_CONFIG;
  std::lock_guard<std::mutex> lk(m->mu);
  m->prog.graph.kernel_policy = policy;
  for (ExecCtx* c : m->all_ctxs) {
    for (auto& cg : c->graphs) cudaGraphExecDestroy(cg.exec);
    c->graphs.clear();
  }
  return ST_OK;
}

// Tensor-core tile configuration of one launch-list step (0 = by shape) and
// whether a following small-N head is fused into its epilogue.  Used by the
// autotuner; call between runs, not concurrently with them.
FTB_API int ftb_model_set_step_config(void* handle, int step, int tc_bn, int tc_bk, int tc_mh, int tc_pair,
                                      int fuse_head) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return ST_NULL;
  if (step < 0 || step >= (int)m->prog.steps.size()) {
    set_error("step index out of range");
    return ST_CONFIG;
  }
  if (!(tc_bn == 0 || tc_bn == 64 || tc_bn == 128 || tc_bn == 256) || !(tc_bk == 0 || tc_bk == 16 || tc_bk == 32) ||
      !(tc_mh >= 0 && tc_mh <= 2) || !(tc_pair >= 0 && tc_pair <= 5)) {
    set_error("tile width must be 0, 64, 128 or 256, k-block 0, 16 or 32, row halves 0, 1 or 2, pair 0..5");
    return ST_CONFIG;
  }
  if (tc_pair >= 2 && tc_pair <= 3 && (tc_mh == 2 || (tc_bn != 0 && tc_bn < 128))) {
    set_error("SM-pair tiles are 256 rows by 128 or 256 columns (row halves 0 or 1)");
    return ST_CONFIG;
  }
  std::lock_guard<std::mutex> lk(m->mu);
  auto apply = [&](Step& s) {
    s.tc_bn = tc_bn;
    s.tc_bk = tc_bk;
    s.tc_mh = tc_mh;
    s.tc_pair = tc_pair;
    s.fuse_head = fuse_head != 0;
  };
  apply(m->prog.steps[(size_t)step]);
  for (auto& rep : m->replicas) apply(rep->steps[(size_t)step]);
  for (ExecCtx* c : m->all_ctxs) {
    for (auto& cg : c->graphs) cudaGraphExecDestroy(cg.exec);
    c->graphs.clear();
  }
  return ST_OK;
}

// Failure-detection hook: while `tc_stall` is non-zero, every tensor-core
// launch of this model first waits on a barrier that nothing completes; the
// bounded wait runs out (about 2 s), the kernel aborts cleanly and the
// synchronous run returns -5.  No fault, trap or unbounded wait is involved.
FTB_API int ftb_model_set_fault_injection(void* handle, int tc_stall) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return ST_NULL;
  m->tc_stall_test.store(tc_stall ? 1 : 0);
  std::lock_guard<std::mutex> lk(m->mu);
  for (ExecCtx* c : m->all_ctxs) {
    for (auto& cg : c->graphs) cudaGraphExecDestroy(cg.exec);
    c->graphs.clear();
  }
  return ST_OK;
}

FTB_API int ftb_model_prepare(void* handle) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return ST_NULL;
  std::vector<int> devs;
  int rc = resolve_devices(m, &devs);
  if (rc) return rc;
  for (int d : devs) {
    Replica* rep = nullptr;
    {
      std::lock_guard<std::mutex> lk(m->mu);
      rc = make_replica(m, d, &rep);
    }
    if (rc) return rc;
    ExecCtx* c = nullptr;
    rc = lease(m, d, &c);
    if (rc) return rc;
    c->in_use = false;
  }
  return ST_OK;
}

FTB_API int ftb_model_run(void* handle, const float* in, size_t in_count, float* out, size_t out_count,
                          int64_t batch, int api) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return ST_NULL;
  int rc = validate(m->prog, in, in_count, out, out_count, &batch, api);
  if (rc) return rc;
  try {
    return run_host(m, in, out, batch);
  } catch (const std::exception& e) {
    set_error(e.what());
    return ST_ALLOC;
  }
}

FTB_API int ftb_model_run_device(void* handle, const float* d_in, size_t in_count, float* d_out, size_t out_count,
                                 int64_t batch, void* stream) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return ST_NULL;
  int rc = validate(m->prog, d_in, in_count, d_out, out_count, &batch, 2);
  if (rc) return rc;
  std::vector<int> devs;
  rc = resolve_devices(m, &devs);
  if (rc) return rc;
  const int dev = devs[0];
  Replica* rep = nullptr;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    rc = make_replica(m, dev, &rep);
  }
  if (rc) return rc;
  ExecCtx* c = nullptr;
  rc = lease(m, dev, &c);
  if (rc) return rc;
  LeaseGuard lg{c};
  DeviceGuard guard(dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);  // NULL: the legacy default stream
  return run_graph(m, rep, c, d_in, d_out, batch, s);
}

static constexpr int kProfSlots = 1024;

// Like ftb_model_run_device, but launches the steps directly (no graph) with
// an event before every step and after the last, kept in `slot` of the
// calling thread's context until ftb_model_profile_read.
FTB_API int ftb_model_run_device_profiled(void* handle, const float* d_in, size_t in_count, float* d_out,
                                          size_t out_count, int64_t batch, void* stream, int slot) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return ST_NULL;
  if (slot < 0 || slot >= kProfSlots) {
    set_error("profile slot out of range");
    return ST_CONFIG;
  }
  int rc = validate(m->prog, d_in, in_count, d_out, out_count, &batch, 2);
  if (rc) return rc;
  std::vector<int> devs;
  rc = resolve_devices(m, &devs);
  if (rc) return rc;
  Replica* rep = nullptr;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    rc = make_replica(m, devs[0], &rep);
  }
  if (rc) return rc;
  ExecCtx* c = nullptr;
  rc = lease(m, devs[0], &c);
  if (rc) return rc;
  LeaseGuard lg{c};
  DeviceGuard guard(devs[0]);
  const size_t per = rep->steps.size() + 1;
  const size_t need = per * (size_t)(slot + 1);
  while (c->prof.size() < need) {
    cudaEvent_t e;
    CUDA_TRY(cudaEventCreate(&e));
    c->prof.push_back(e);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);  // NULL: the legacy default stream
  return enqueue(m, rep, c, d_in, d_out, batch, s, c->prof.data() + per * slot);
}

// Waits for the events of `slot` and writes each step's device time (ms).
// Returns the number of steps, or a negative status.
FTB_API int ftb_model_profile_read(void* handle, int slot, float* step_ms, int cap) {
  auto* m = static_cast<Model*>(handle);
  if (!m || !step_ms) return ST_NULL;
  std::vector<int> devs;
  int rc = resolve_devices(m, &devs);
  if (rc) return rc;
  ExecCtx* c = nullptr;
  rc = lease(m, devs[0], &c);
  if (rc) return rc;
  LeaseGuard lg{c};
  DeviceGuard guard(devs[0]);
  const size_t n = m->prog.steps.size();
  const size_t per = n + 1;
  if (slot < 0 || per * (size_t)(slot + 1) > c->prof.size()) {
    set_error("profile slot was never recorded on this thread");
    return ST_CONFIG;
  }
  for (size_t i = 0; i < n && (int)i < cap; ++i) {
    CUDA_TRY(cudaEventSynchronize(c->prof[per * slot + i + 1]));
    float ms = 0.0f;
    CUDA_TRY(cudaEventElapsedTime(&ms, c->prof[per * slot + i], c->prof[per * slot + i + 1]));
    step_ms[i] = ms;
  }
  return (int)n;
}

FTB_API double ftb_model_benchmark(void* handle, const float* in, size_t in_count, float* out, size_t out_count,
                                   int iters) {
  auto* m = static_cast<Model*>(handle);
  if (!m || !in || !out || iters <= 0) return -1.0;
  const Program& p = m->prog;
  int64_t batch;
  if (p.dynamic) {
    const int64_t si = p.in_static_elems;
    if (si == 0 || in_count == 0 || in_count % (size_t)si != 0) return -2.0;
    batch = (int64_t)(in_count / (size_t)si);
    if (batch <= 0 || batch > p.max_batch) return -2.0;
    const size_t want_out = p.output_dynamic ? (size_t)(batch * p.out_static_elems) : (size_t)p.out_static_elems;
    if (out_count != want_out) return -3.0;
  } else {
    if (in_count != (size_t)p.in_static_elems) return -2.0;
    if (out_count != (size_t)p.out_static_elems) return -3.0;
    batch = p.static_batch;
  }
  std::vector<int> devs;
  if (resolve_devices(m, &devs)) return -4.0;
  const int dev = devs[0];
  Replica* rep = nullptr;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    if (make_replica(m, dev, &rep)) return -4.0;
  }
  ExecCtx* c = nullptr;
  if (lease(m, dev, &c)) return -4.0;
  LeaseGuard lg{c};
  DeviceGuard guard(dev);
  const size_t in_b = in_count * 4, out_b = out_count * 4;
  if (cudaMemcpyAsync(c->d_in, in, in_b, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) return -5.0;
  for (int w = 0; w < 10; ++w)
    if (run_graph(m, rep, c, c->d_in, c->d_out, batch, c->stream)) return -5.0;
  if (cudaEventRecord(c->ev_a, c->stream) != cudaSuccess) return -5.0;
  for (int i = 0; i < iters; ++i)
    if (run_graph(m, rep, c, c->d_in, c->d_out, batch, c->stream)) return -5.0;
  if (cudaEventRecord(c->ev_b, c->stream) != cudaSuccess) return -5.0;
  if (cudaMemcpyAsync(out, c->d_out, out_b, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -5.0;
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return -5.0;
  float ms = 0.0f;
  if (cudaEventElapsedTime(&ms, c->ev_a, c->ev_b) != cudaSuccess) return -5.0;
  return (double)ms * 1000.0 / iters;
}

FTB_API int ftb_model_is_dynamic(void* handle) {
  auto* m = static_cast<Model*>(handle);
  return m && m->prog.dynamic ? 1 : 0;
}

FTB_API int64_t ftb_model_max_batch(void* handle) {
  auto* m = static_cast<Model*>(handle);
  return m ? m->prog.max_batch : 0;
}

// which: 0 total (payload + insertions), 1 payload, 2 insertions, 3 process total
FTB_API size_t ftb_model_counter(void* handle, int which) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return 0;
  if (which == 3) return m->process_allocs.load();
  if (which == 4) return m->graph_kernels.load();
  size_t payload = 0, ins = 0;
  for (auto& kv : t_pools.pools)
    if (kv.first.uid == m->uid) {
      payload += kv.second.payload_allocs;
      ins += kv.second.block_insertions;
    }
  return which == 1 ? payload : which == 2 ? ins : payload + ins;
}

FTB_API void ftb_model_reset_counters(void* handle) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return;
  for (auto& kv : t_pools.pools)
    if (kv.first.uid == m->uid) {
      kv.second.payload_allocs = 0;
      kv.second.block_insertions = 0;
    }
}

// Forces a 64 MiB arena allocation in this thread's pool (the reference's
// forgetune_test_inject_arena_alloc, src/codegen.cpp:1125-1130).
FTB_API void ftb_model_inject_alloc(void* handle) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return;
  std::vector<int> devs;
  if (resolve_devices(m, &devs)) return;
  ExecCtx* c = nullptr;
  if (lease(m, devs[0], &c)) return;
  LeaseGuard lg{c};
  DeviceGuard guard(c->device);
  if (layout_block(m, c, c->block_bytes + (64u << 20), nullptr) == ST_OK) {
    pool_of(m, devs[0]).payload_allocs++;
    m->process_allocs++;
  }
}

FTB_API int ftb_model_describe(void* handle, char* buf, size_t cap) {
  auto* m = static_cast<Model*>(handle);
  if (!m) return ST_NULL;
  std::string s = m->prog.describe();
  if (buf && cap) {
    size_t n = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return (int)s.size();
}

FTB_API int ftb_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Elements [first, first+count) of the Philox4x32-10 normal stream keyed by
// seed, written to device memory d_out on `stream`.
FTB_API int ftb_philox_normal(float* d_out, uint64_t seed, uint64_t first, uint64_t count, void* stream) {
  if (!d_out) return ST_NULL;
  if (count == 0) return ST_OK;
  int dev = 0, sm = 148;
  CUDA_TRY(cudaGetDevice(&dev));
  cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t blocks = (count + 3) / 4 + 1;
  const unsigned grid = (unsigned)std::min<uint64_t>((blocks + 255) / 256, (uint64_t)sm * 16);
  philox_normal_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_out, seed, first, count);
  CUDA_TRY(cudaGetLastError());
  return ST_OK;
}

// ===========================================================================
// Split-K GEMM for up to 16 rows that allocates nothing
// ===========================================================================
// Some callers cannot allocate device memory where they call us: a plugin
// running inside another engine's execution step (an inference server or
// graph runtime that owns all device memory and forbids allocation there), or
// a latency-critical loop that cannot afford cudaMalloc's implicit device
// synchronisation.  ftb_small_gemm_noalloc gives them the split-K kernel with
// its scratch -- the slice partial sums and the per-column-block tickets -- in
// one file-scope __device__ array of fixed size instead of a context arena.
// Every GPU on which this library's module is loaded holds that array
// (4 MiB + 4 KiB) until the process exits.  All calls on a device share it and
// it keeps the previous call's partial sums; the tickets, which must start at
// zero, are cleared by every call.  Calls that overlap on the GPU (unordered
// streams) race on the shared array.
namespace ftb {
constexpr size_t kNoAllocPartFloats = size_t(1) << 20;  // 4 MiB of partial sums
constexpr int kNoAllocTickets = 1024;                    // N up to 65536
struct NoAllocScratch {
  float part[kNoAllocPartFloats];
  unsigned tickets[kNoAllocTickets];
};
}  // namespace ftb

static __device__ __align__(256) ftb::NoAllocScratch g_noalloc_scratch;

namespace ftb {
constexpr int kNoAllocMaxDevices = 64;
struct NoAllocDevice {
  std::once_flag once;
  int rc = ST_OK;
  std::string err;
  NoAllocScratch* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int sm_count = 0;
};
static NoAllocDevice g_noalloc_devices[kNoAllocMaxDevices];

// One-time set-up for `dev`, which is the current device: the device address
// of the scratch array (in host code the array's name is only a host-side
// stand-in) and the shared-memory attribute of the kernels it launches.
static void noalloc_setup(int dev, NoAllocDevice* d) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) {
    d->rc = ST_DEVICE;
    d->err = std::string("cudaGetSymbolAddress of the split-K scratch failed: ") + cudaGetErrorString(e);
    cudaGetLastError();
    return;
  }
  d->scratch = static_cast<NoAllocScratch*>(p);
  e = cudaDeviceGetAttribute(&d->sm_count, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(splitk_gemv_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(splitk_gemv_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
  if (e != cudaSuccess) {
    d->rc = ST_DEVICE;
    d->err = std::string("split-K kernel set-up failed: ") + cudaGetErrorString(e);
    cudaGetLastError();
  }
}
}  // namespace ftb

FTB_API int ftb_small_gemm_noalloc(const float* d_x, const float* d_w, const float* d_bias, const float* d_residual,
                                   float* d_y, int64_t m, int64_t k, int64_t n, uint32_t flags, void* stream) {
  if (!d_x || !d_w || !d_y) return ST_NULL;
  if (((flags & FTB_SMALL_GEMM_BIAS) && !d_bias) || ((flags & FTB_SMALL_GEMM_RESIDUAL) && !d_residual))
    return ST_NULL;
  if (m < 1 || m > 16 || k < 1 || n < 1 || k > (1 << 30) || n > (1 << 30)) {
    set_error("ftb_small_gemm_noalloc: needs 1 <= m <= 16 and positive k, n");
    return ST_INPUT;
  }
  if ((flags & FTB_SMALL_GEMM_RESIDUAL) && k != n) {
    set_error("ftb_small_gemm_noalloc: a residual needs k == n");
    return ST_INPUT;
  }
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    set_error("ftb_small_gemm_noalloc: device ordinal beyond the supported range");
    return ST_CONFIG;
  }
  NoAllocDevice& d = g_noalloc_devices[dev];
  std::call_once(d.once, [&]() { noalloc_setup(dev, &d); });
  if (d.rc != ST_OK) {
    set_error(d.err);
    return d.rc;
  }
  int ks = 0, kc = 0;
  splitk_shape(k, n, d.sm_count, &ks, &kc);
  const size_t need = (size_t)ks * 16 * (size_t)n;
  const int64_t blocks = (n + kSkCols - 1) / kSkCols;
  if (need > kNoAllocPartFloats || blocks > kNoAllocTickets) {
    set_error("ftb_small_gemm_noalloc: k=" + std::to_string(k) + ", n=" + std::to_string(n) + " needs " +
              std::to_string(need) + " floats of partial sums; the fixed scratch holds " +
              std::to_string(kNoAllocPartFloats));
    return ST_INPUT;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaMemsetAsync(d.scratch->tickets, 0, sizeof(unsigned) * (size_t)blocks, s));
  SplitKArgs a{};
  a.A = d_x;
  a.B = d_w;
  a.bias = d_bias;
  a.res = d_residual;
  a.Y = d_y;
  a.part = d.scratch->part;
  a.tickets = d.scratch->tickets;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.epi = ((flags & FTB_SMALL_GEMM_BIAS) ? EPI_BIAS_LAST : 0u) | ((flags & FTB_SMALL_GEMM_RELU) ? EPI_RELU_PRE : 0u) |
          ((flags & FTB_SMALL_GEMM_RESIDUAL) ? EPI_RESIDUAL : 0u);
  cudaError_t lerr = cudaSuccess;
  const int rc = launch_splitk(a, d.sm_count, s, &lerr);
  if (rc != 0) {
    set_error(std::string("ftb_small_gemm_noalloc: launch failed: ") + cudaGetErrorString(lerr));
    return ST_DEVICE;
  }
  return ST_OK;
}

// ---------------------------------------------------------------------------
// Tuned kernel table and device description (autotuner)
// ---------------------------------------------------------------------------
FTB_API int ftb_model_set_tuning(void* handle, const int64_t* records, int n) {
  auto* m = static_cast<Model*>(handle);
  if (!m || (n > 0 && !records)) {
    set_error("null model or records");
    return ST_NULL;
  }
  if (n < 0 || n > (1 << 16)) {
    set_error("record count out of range");
    return ST_CONFIG;
  }
  std::vector<TuneRecord> recs((size_t)n);
  for (int i = 0; i < n; ++i) {
    const int64_t* w = records + (size_t)i * kTuneWords;
    TuneRecord& r = recs[(size_t)i];
    r.step = w[0];
    r.batch_lo = w[1];
    r.batch_hi = w[2];
    r.family = (int32_t)w[3];
    r.bn = (int32_t)w[4];
    r.bk = (int32_t)w[5];
    r.mh = (int32_t)w[6];
    r.pair = (int32_t)w[7];
    r.fuse_head = w[8] != 0;
  }
  std::lock_guard<std::mutex> lk(m->mu);
  try {
    apply_tuning(m->prog.steps, recs);
    for (auto& rep : m->replicas) apply_tuning(rep->steps, recs);
  } catch (const std::exception& e) {
    set_error(e.what());
    return ST_CONFIG;
  }
  for (ExecCtx* c : m->all_ctxs) {
    for (auto& cg : c->graphs) cudaGraphExecDestroy(cg.exec);
    c->graphs.clear();
  }
  return ST_OK;
}

FTB_API int ftb_device_info(int device, char* buf, size_t cap) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    set_error(std::string("no CUDA device ") + std::to_string(device));
    return ST_DEVICE;
  }
  int drv = 0, rt = 0;
  cudaDriverGetVersion(&drv);
  cudaRuntimeGetVersion(&rt);
  std::string name(prop.name);
  for (char& ch : name)
    if (ch == '"' || ch == '\\') ch = ' ';
  const std::string js = "{\"name\":\"" + name + "\",\"cc\":\"" + std::to_string(prop.major) + "." +
                         std::to_string(prop.minor) + "\",\"sm_count\":" + std::to_string(prop.multiProcessorCount) +
                         ",\"memory_bytes\":" + std::to_string((unsigned long long)prop.totalGlobalMem) +
                         ",\"driver_version\":" + std::to_string(drv) + ",\"runtime_version\":" + std::to_string(rt) +
                         "}";
  if (buf && cap > 0) {
    const size_t k = std::min(cap - 1, js.size());
    std::memcpy(buf, js.data(), k);
    buf[k] = 0;
  }
  return (int)js.size();
}
