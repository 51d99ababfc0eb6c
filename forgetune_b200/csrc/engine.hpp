// Host-side engine: graph blob, fusion, arena planning and launch plan.
//
// The graph arrives as a flat little-endian blob written by
// forgetune_b200/graph_blob.py (the compile step).  It carries the
// reference IR after export -- INPUT / CONST / MATMUL / ADD / RELU / MUL /
// SIGMOID / TANH / CONV2D / FLATTEN nodes in topological order
// (include/forgetune/ir.hpp:162-177 of the reference) -- plus the weights.
// The engine then
//   1. fuses, following src/fusion.cpp:6-131 of the reference
//      (MATMUL->ADD->RELU, CONV2D->RELU), and additionally folds the bias
//      ADD, the residual ADD and a trailing RELU into the GEMM epilogue and
//      turns FLATTEN into a view;
//   2. plans one device arena with the reference's greedy lowest-offset
//      interval colouring (src/memory_planner.cpp:33-174), sized at
//      max_batch;
//   3. emits a launch list (Step) that the CUDA runtime replays.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "flags.h"

namespace ftb {

enum OpKind : int32_t {
  OP_INPUT = 0,
  OP_CONST = 1,
  OP_MATMUL = 2,
  OP_ADD = 3,
  OP_RELU = 4,
  OP_OUTPUT = 5,
  OP_FUSED_MATMUL_ADD_RELU = 6,
  OP_MUL = 7,
  OP_SIGMOID = 8,
  OP_TANH = 9,
  OP_CONV2D = 10,
  OP_FLATTEN = 11,
  OP_FUSED_CONV2D_RELU = 12,
  // engine-internal, produced by fusion only
  OP_GEMM = 100,  // x.W with an epilogue (bias / relu / residual / relu)
  OP_CONV = 101,  // implicit-GEMM conv with an epilogue
};

const char* op_name(int32_t op);

constexpr int64_t kDynamicDim = -1;

struct Shape {
  int32_t rank = 0;
  int64_t dims[4] = {0, 0, 0, 0};
  bool dynamic() const { return rank > 0 && dims[0] == kDynamicDim; }
  // elements per leading-batch row (product of dims[1:]) for dynamic shapes,
  // or the full element count for static ones
  int64_t static_elems() const;
  int64_t elems(int64_t batch) const;  // reference TensorShape::element_count
};

struct ConvAttrs {
  int64_t sh = 1, sw = 1, ph = 0, pw = 0, dh = 1, dw = 1;
};

struct Node {
  int32_t id = -1;
  int32_t op = OP_INPUT;
  std::vector<int32_t> inputs;
  Shape shape;
  ConvAttrs conv;
  uint64_t const_offset = 0;  // floats into the weight section
  uint64_t const_count = 0;
  bool deleted = false;
  // filled by fusion for OP_GEMM / OP_CONV
  uint32_t epi = 0;
  int32_t bias_id = -1;
  int32_t residual_id = -1;
  int32_t alias_of = -1;  // FLATTEN as a view of this node's buffer
};

// Compile options carried in the blob header.
enum BlobFlags : uint32_t {
  BLOB_DYNAMIC = 1u << 0,
  BLOB_FUSION = 1u << 1,          // reference fusion pass enabled
  BLOB_BIAS_FIRST_FUSED = 1u << 2,  // fused_ikj / loop_ikj order for fused nodes
  BLOB_NO_FOLD = 1u << 3,           // reference fusion only: no epilogue folding, FLATTEN copies
};

enum KernelPolicy : int32_t {
  KP_AUTO = 0,        // tcgen05 3xTF32 for large dense GEMMs, SIMT FFMA otherwise
  KP_SIMT = 1,        // SIMT FFMA everywhere
  KP_SIMT_EXACT = 2,  // SIMT with separately rounded mul + add in the reference's order
  KP_TCGEN05 = 3,     // tcgen05 wherever the shape allows it
};

// One entry of a tuned kernel table: for launch-list step `step` and a
// per-replica batch in [batch_lo, batch_hi], run this kernel family and
// tile configuration (written by the autotuner, carried in the graph blob).
enum TuneFamily : int32_t {
  TF_HEURISTIC = 0,  // the engine's shape rules
  TF_SIMT = 1,       // SIMT FFMA GEMM
  TF_SPLITK = 2,     // split-K GEMV (batch rows <= 16)
  TF_TCGEN05 = 3,    // tensor cores
};
constexpr int kTuneWords = 9;  // step, batch_lo, batch_hi, family, bn, bk, mh, pair, fuse_head
struct TuneRecord {
  int64_t step = 0, batch_lo = 1, batch_hi = 0;
  int32_t family = TF_HEURISTIC, bn = 0, bk = 0, mh = 0, pair = 0;
  bool fuse_head = true;
};
// Checks one record's values (not the step index); "" when valid.
std::string check_tune_record(const TuneRecord& r);

struct Graph {
  std::vector<Node> nodes;  // index == id
  int32_t input_id = -1;
  int32_t output_id = -1;
  int64_t max_batch = 128;
  uint32_t flags = 0;
  int32_t kernel_policy = KP_AUTO;
  int64_t static_batch = 1;
  std::vector<float> weights;
  std::vector<TuneRecord> tuning;  // optional trailer of the blob

  const Node& node(int32_t id) const { return nodes.at(static_cast<size_t>(id)); }
  Node& node(int32_t id) { return nodes.at(static_cast<size_t>(id)); }
  std::vector<int32_t> order() const;  // live nodes in blob (topological) order
  std::vector<int> use_counts() const;
};

// Parse + validate; throws std::runtime_error with a message on malformed input.
Graph parse_blob(const void* data, size_t bytes);

// Reference fusion (src/fusion.cpp) when `reference_fusion`, then epilogue
// folding (bias / residual / trailing ReLU, FLATTEN views) when `fold`.
void fuse(Graph& g, bool reference_fusion, bool fold);

struct Alloc {
  int32_t node_id = -1;
  size_t offset = 0;
  size_t size_bytes = 0;
  int birth = 0;
  int death = 0;
};

struct ArenaPlan {
  size_t arena_bytes = 0;
  size_t naive_bytes = 0;
  size_t peak_live_bytes = 0;
  double savings_percent = 0.0;
  std::vector<Alloc> allocs;  // in execution order
  const Alloc* find(int32_t id) const;
};

// Greedy lowest-offset interval colouring (src/memory_planner.cpp:33-174).
ArenaPlan plan_arena(const Graph& g, int64_t max_batch, size_t alignment);

// Where an operand lives at run time.
enum Space : int32_t { SP_NONE = 0, SP_INPUT = 1, SP_OUTPUT = 2, SP_ARENA = 3, SP_WEIGHT = 4 };

struct Operand {
  int32_t space = SP_NONE;
  uint64_t offset = 0;  // bytes into the arena, or floats into the device weights
};

enum StepKind : int32_t {
  ST_GEMM = 0,
  ST_CONV = 1,
  ST_ADD_SAME = 2,
  ST_ADD_ROW = 3,
  ST_ADD_CHANNEL = 4,
  ST_MUL_SAME = 5,
  ST_MUL_ROW = 6,
  ST_MUL_CHANNEL = 7,
  ST_RELU = 8,
  ST_SIGMOID = 9,
  ST_TANH = 10,
  ST_COPY = 11,
  ST_FILL_CONST = 12,  // graph output that is a constant
};

struct Step {
  int32_t kind = ST_GEMM;
  int32_t node_id = -1;
  Operand a, b, bias, res, out;
  uint32_t epi = 0;
  // GEMM: y[M,N] = x[M,K] W[K,N]; rows M = batch * rows_per_sample
  int64_t K = 0, N = 0;
  int64_t rows_per_sample = 1;
  // conv geometry
  int64_t Cin = 0, H = 0, W = 0, Cout = 0, Kh = 0, Kw = 0, Ho = 0, Wo = 0;
  ConvAttrs conv;
  // elementwise: elements per sample (or per batch for static operands)
  int64_t elems_per_sample = 0;
  int64_t row_len = 0;   // ADD_ROW / MUL_ROW width
  int64_t channels = 0;  // ADD_CHANNEL: C, HW in row_len
  bool static_rows = false;  // operand is not batch-dependent
  // device weight-layout slots, filled at upload: W[K,N] for SIMT,
  // W^T split into tf32 hi / lo [N,Kp] for the tensor-core path
  uint64_t w_kn = 0, w_nk_hi = 0, w_nk_lo = 0;
  uint64_t w_nk_f32 = 0;  // fp32 W^T [N, K] for the small-batch chain kernel (0 = none)
  int64_t Kp = 0;  // K padded to the tensor-core k-block
  // Small-N head: the GEMM step right after this one consumes only this
  // step's output and has N <= kMaxHeadN, so a tensor-core launch of this
  // step can compute it in its epilogue (the intermediate is never stored).
  int32_t head_step = -1;  // index of that step, or -1
  int32_t head_of = -1;    // on the head step: the step that may absorb it
  // Two-layer fusion: the GEMM step right after this one consumes only this
  // step's output, 128 < N <= 256 here and 64 <= N <= 128 there, epilogues of
  // column biases and ReLUs: one kernel may compute both layers (and the
  // second one's head) with this step's output kept in tensor memory.
  int32_t mlp_step = -1;   // index of that step, or -1
  int32_t mlp_of = -1;     // on that step: the step that may absorb it
  // tensor-core tile configuration chosen for this step (0 = by shape), and
  // whether a head may be fused (set by the autotuner or the caller)
  int32_t tc_bn = 0;
  int32_t tc_bk = 0;
  int32_t tc_mh = 0;  // 128-row halves per tile (0 = by shape)
  int32_t tc_pair = 0;  // 2 = 256-row tiles on an SM pair, 1 = one SM per tile, 3 = pair with split-K,
                        // 4 = this layer and the next in one kernel (mlp_step); 0 = by shape
  bool fuse_head = true;
  // tuned choices by batch range (GEMM steps); the first matching entry wins
  std::vector<TuneRecord> tuned;
  const TuneRecord* tuned_for(int64_t batch) const {
    for (const auto& r : tuned)
      if (batch >= r.batch_lo && batch <= r.batch_hi) return &r;
    return nullptr;
  }
};

constexpr int64_t kMaxHeadN = 16;
constexpr int64_t kMaxHeadK = 256;
constexpr int64_t kMlpMinN1 = 129, kMlpMaxN1 = 256, kMlpMinN2 = 64, kMlpMaxN2 = 128;

struct Program {
  Graph graph;
  ArenaPlan plan;
  std::vector<Step> steps;
  int64_t in_static_elems = 0;   // per-sample input floats (dynamic) or total
  int64_t out_static_elems = 0;  // per-sample output floats (dynamic) or total
  bool dynamic = false;
  bool output_dynamic = false;
  int64_t static_batch = 1;
  int64_t max_batch = 128;
  std::string describe() const;  // JSON, for tests and manifests
};

// parse -> fuse -> plan -> steps (and the blob's tuning records onto their steps)
Program build_program(const void* blob, size_t bytes);

// Replaces the tuned tables of `steps` with `records`; throws
// std::runtime_error naming the first invalid record.
void apply_tuning(std::vector<Step>& steps, const std::vector<TuneRecord>& records);

}  // namespace ftb
