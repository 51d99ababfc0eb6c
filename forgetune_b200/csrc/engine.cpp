// Host-side engine: blob parsing, fusion, arena planning, launch list.
#include "engine.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <sstream>
#include <stdexcept>
#include <unordered_map>
#include <unordered_set>

namespace ftb {

const char* op_name(int32_t op) {
  switch (op) {
    case OP_INPUT: return "INPUT";
    case OP_CONST: return "CONST";
    case OP_MATMUL: return "MATMUL";
    case OP_ADD: return "ADD";
    case OP_RELU: return "RELU";
    case OP_OUTPUT: return "OUTPUT";
    case OP_FUSED_MATMUL_ADD_RELU: return "FUSED_MATMUL_ADD_RELU";
    case OP_MUL: return "MUL";
    case OP_SIGMOID: return "SIGMOID";
    case OP_TANH: return "TANH";
    case OP_CONV2D: return "CONV2D";
    case OP_FLATTEN: return "FLATTEN";
    case OP_FUSED_CONV2D_RELU: return "FUSED_CONV2D_RELU";
    case OP_GEMM: return "GEMM";
    case OP_CONV: return "CONV";
    default: return "UNKNOWN";
  }
}

int64_t Shape::static_elems() const {
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) {
    if (i == 0 && dims[0] == kDynamicDim) continue;
    n *= dims[i];
  }
  return n;
}

int64_t Shape::elems(int64_t batch) const {
  if (rank == 0) return 1;
  return dynamic() ? batch * static_elems() : static_elems();
}

static bool same_shape(const Shape& a, const Shape& b) {
  if (a.rank != b.rank) return false;
  for (int i = 0; i < a.rank; ++i)
    if (a.dims[i] != b.dims[i]) return false;
  return true;
}

std::vector<int32_t> Graph::order() const {
  std::vector<int32_t> o;
  for (const auto& n : nodes)
    if (!n.deleted && n.id >= 0) o.push_back(n.id);
  return o;
}

std::vector<int> Graph::use_counts() const {
  std::vector<int> uc(nodes.size(), 0);
  for (const auto& n : nodes) {
    if (n.deleted || n.id < 0) continue;
    for (int32_t in : n.inputs) uc.at(static_cast<size_t>(in))++;
  }
  return uc;
}

// ---------------------------------------------------------------------------
// blob
// ---------------------------------------------------------------------------
static constexpr char kMagicText[8] = {'F', 'T', 'B', 'G', 'R', 'A', 'P', 'H'};
static constexpr int64_t kVersion = 1;
static constexpr int kHeaderWords = 12;
static constexpr int kNodeWords = 20;
// optional trailer after the weights (8-byte aligned): magic, record count,
// then kTuneWords int64 per record
static constexpr char kTuneMagic[8] = {'F', 'T', 'B', 'T', 'U', 'N', 'E', '1'};

std::string check_tune_record(const TuneRecord& r) {
  if (r.batch_lo < 1 || r.batch_hi < r.batch_lo) return "batch range must satisfy 1 <= lo <= hi";
  if (r.family < TF_HEURISTIC || r.family > TF_TCGEN05) return "family must be 0..3";
  if (!(r.bn == 0 || r.bn == 64 || r.bn == 128 || r.bn == 256)) return "tile width must be 0, 64, 128 or 256";
  if (!(r.bk == 0 || r.bk == 16 || r.bk == 32)) return "k-block must be 0, 16 or 32";
  if (r.mh < 0 || r.mh > 2) return "row halves must be 0, 1 or 2";
  if (r.pair < 0 || r.pair > 5) return "pair must be 0, 1, 2, 3, 4 or 5";
  if (r.pair >= 2 && r.pair <= 3 && (r.mh == 2 || (r.bn != 0 && r.bn < 128))) return "SM-pair tiles need width 0, 128 or 256 and row halves 0 or 1";
  return "";
}

Graph parse_blob(const void* data, size_t bytes) {
  if (!data || bytes < kHeaderWords * 8) throw std::runtime_error("graph blob too small");
  const auto* base = static_cast<const uint8_t*>(data);
  int64_t h[kHeaderWords];
  std::memcpy(h, base, sizeof(h));
  if (std::memcmp(base, kMagicText, 8) != 0) throw std::runtime_error("graph blob: bad magic");
  if (h[1] != kVersion) throw std::runtime_error("graph blob: unsupported version");
  Graph g;
  const int64_t n_nodes = h[2];
  g.input_id = static_cast<int32_t>(h[3]);
  g.output_id = static_cast<int32_t>(h[4]);
  g.max_batch = h[5];
  g.flags = static_cast<uint32_t>(h[6]);
  g.kernel_policy = static_cast<int32_t>(h[7]);
  g.static_batch = h[8];
  const uint64_t n_w = static_cast<uint64_t>(h[9]);
  const uint64_t nodes_off = static_cast<uint64_t>(h[10]);
  const uint64_t w_off = static_cast<uint64_t>(h[11]);
  if (n_nodes <= 0 || n_nodes > (1 << 20)) throw std::runtime_error("graph blob: bad node count");
  if (nodes_off + static_cast<uint64_t>(n_nodes) * kNodeWords * 8 > bytes)
    throw std::runtime_error("graph blob: node table out of range");
  if (w_off > bytes || n_w > (bytes - w_off) / 4) throw std::runtime_error("graph blob: weights out of range");
  if (g.max_batch <= 0 || g.max_batch > 1000000) throw std::runtime_error("graph blob: max_batch out of [1, 1000000]");
  g.nodes.resize(static_cast<size_t>(n_nodes));
  for (int64_t i = 0; i < n_nodes; ++i) {
    int64_t r[kNodeWords];
    std::memcpy(r, base + nodes_off + static_cast<uint64_t>(i) * kNodeWords * 8, sizeof(r));
    Node n;
    n.id = static_cast<int32_t>(r[0]);
    if (n.id != i) throw std::runtime_error("graph blob: node ids must be dense and ordered");
    n.op = static_cast<int32_t>(r[1]);
    const int64_t nin = r[2];
    if (nin < 0 || nin > 4) throw std::runtime_error("graph blob: bad input count");
    for (int64_t k = 0; k < nin; ++k) {
      const int64_t in = r[3 + k];
      if (in < 0 || in >= i) throw std::runtime_error("graph blob: inputs must precede their consumer");
      n.inputs.push_back(static_cast<int32_t>(in));
    }
    n.shape.rank = static_cast<int32_t>(r[7]);
    if (n.shape.rank < 0 || n.shape.rank > 4) throw std::runtime_error("graph blob: rank must be 0..4");
    for (int k = 0; k < 4; ++k) n.shape.dims[k] = r[8 + k];
    for (int k = 0; k < n.shape.rank; ++k)
      if (n.shape.dims[k] <= 0 && !(k == 0 && n.shape.dims[k] == kDynamicDim))
        throw std::runtime_error("graph blob: non-positive dimension");
    n.conv.sh = r[12]; n.conv.sw = r[13]; n.conv.ph = r[14];
    n.conv.pw = r[15]; n.conv.dh = r[16]; n.conv.dw = r[17];
    n.const_offset = static_cast<uint64_t>(r[18]);
    n.const_count = static_cast<uint64_t>(r[19]);
    if (n.op == OP_CONST) {
      if (n.const_offset + n.const_count > n_w) throw std::runtime_error("graph blob: constant out of range");
      if (static_cast<int64_t>(n.const_count) != n.shape.elems(1))
        throw std::runtime_error("graph blob: constant size does not match its shape");
    }
    g.nodes[static_cast<size_t>(i)] = n;
  }
  if (g.input_id < 0 || g.input_id >= n_nodes || g.nodes[g.input_id].op != OP_INPUT)
    throw std::runtime_error("graph blob: graph must have exactly one INPUT");
  if (g.output_id < 0 || g.output_id >= n_nodes) throw std::runtime_error("graph blob: bad output id");
  g.weights.resize(n_w);
  if (n_w) std::memcpy(g.weights.data(), base + w_off, n_w * 4);
  const uint64_t t_off = (w_off + n_w * 4 + 7) / 8 * 8;
  if (t_off + 16 <= bytes && std::memcmp(base + t_off, kTuneMagic, 8) == 0) {
    int64_t n_rec = 0;
    std::memcpy(&n_rec, base + t_off + 8, 8);
    if (n_rec < 0 || n_rec > 1 << 16 || t_off + 16 + static_cast<uint64_t>(n_rec) * kTuneWords * 8 > bytes)
      throw std::runtime_error("graph blob: tuning table out of range");
    for (int64_t i = 0; i < n_rec; ++i) {
      int64_t w[kTuneWords];
      std::memcpy(w, base + t_off + 16 + static_cast<uint64_t>(i) * kTuneWords * 8, sizeof(w));
      TuneRecord r;
      r.step = w[0];
      r.batch_lo = w[1];
      r.batch_hi = w[2];
      r.family = static_cast<int32_t>(w[3]);
      r.bn = static_cast<int32_t>(w[4]);
      r.bk = static_cast<int32_t>(w[5]);
      r.mh = static_cast<int32_t>(w[6]);
      r.pair = static_cast<int32_t>(w[7]);
      r.fuse_head = w[8] != 0;
      const std::string why = check_tune_record(r);
      if (!why.empty()) throw std::runtime_error("graph blob: tuning record " + std::to_string(i) + ": " + why);
      g.tuning.push_back(r);
    }
  }
  for (float v : g.weights)
    if (!std::isfinite(v)) throw std::runtime_error("graph blob: non-finite constant");
  return g;
}

// ---------------------------------------------------------------------------
// fusion
// ---------------------------------------------------------------------------
static bool is_bias_vector(const Shape& s, int64_t N) {
  if (s.rank == 1) return s.dims[0] == N;
  if (s.rank == 2) return s.dims[0] == 1 && s.dims[1] == N;
  return false;
}

static bool is_bias_rows(const Shape& s) {
  return s.rank == 2 && (s.dims[0] > 1 || s.dims[0] == kDynamicDim);
}

// Writes the fused op into the consumer's slot: it keeps the consumer's id
// (so its users need no rewiring), shape and execution position.
static void become(Graph& g, int32_t dst, Node fused) {
  fused.id = dst;
  Node& d = g.node(dst);
  fused.shape = d.shape;
  d = fused;
}

void fuse(Graph& g, bool reference_fusion, bool fold) {
  const bool bias_first = (g.flags & BLOB_BIAS_FIRST_FUSED) != 0;
  // Pass 1: the reference patterns, to a fixed point (src/fusion.cpp:6-131).
  bool changed = reference_fusion;
  while (changed) {
    changed = false;
    auto uc = g.use_counts();
    for (auto& r : g.nodes) {
      if (r.deleted || r.op != OP_RELU || r.inputs.size() != 1) continue;
      const int32_t in_id = r.inputs[0];
      Node& in = g.node(in_id);
      if (in.deleted) continue;
      if (in.op == OP_CONV2D) {
        if (uc[in_id] != 1 || in_id == g.output_id) continue;
        Node f;
        f.op = OP_CONV;
        f.inputs = in.inputs;
        f.conv = in.conv;
        f.epi = EPI_RELU_PRE;
        if (in.inputs.size() == 3) {
          f.bias_id = in.inputs[2];
          f.epi |= EPI_BIAS_FIRST;
        }
        in.deleted = true;
        become(g, r.id, f);
        changed = true;
        break;
      }
      if (in.op != OP_ADD || in.inputs.size() != 2) continue;
      if (uc[in_id] != 1 || in_id == g.output_id) continue;
      int32_t mm_id = -1, b_id = -1;
      if (g.node(in.inputs[0]).op == OP_MATMUL) {
        mm_id = in.inputs[0];
        b_id = in.inputs[1];
      } else if (g.node(in.inputs[1]).op == OP_MATMUL) {
        mm_id = in.inputs[1];
        b_id = in.inputs[0];
      } else {
        continue;
      }
      Node& mm = g.node(mm_id);
      if (mm.deleted || mm.inputs.size() != 2) continue;
      if (uc[mm_id] != 1 || mm_id == g.output_id) continue;
      Node f;
      f.op = OP_GEMM;
      f.inputs = {mm.inputs[0], mm.inputs[1], b_id};
      f.bias_id = b_id;
      f.epi = (bias_first ? EPI_BIAS_FIRST : EPI_BIAS_LAST) | EPI_RELU_PRE;
      if (is_bias_rows(g.node(b_id).shape)) f.epi |= EPI_BIAS_ROWS;
      mm.deleted = true;
      in.deleted = true;
      become(g, r.id, f);
      changed = true;
      break;
    }
  }
  // FUSED nodes outside the reference patterns: plain MATMUL / CONV2D.
  for (auto& n : g.nodes) {
    if (n.deleted) continue;
    if (n.op == OP_MATMUL) {
      n.op = OP_GEMM;
      n.epi = 0;
    } else if (n.op == OP_CONV2D) {
      n.op = OP_CONV;
      n.epi = 0;
      if (n.inputs.size() == 3) {
        n.bias_id = n.inputs[2];
        n.epi |= EPI_BIAS_FIRST;
      }
    }
  }
  if (!fold) return;

  // Pass 2: fold bias ADD, residual ADD and a trailing RELU into GEMM
  // epilogues; make FLATTEN a view.  Every fold keeps the reference's
  // arithmetic: ((sum + b) [relu]) + r [relu], each a separately rounded op.
  changed = true;
  while (changed) {
    changed = false;
    auto uc = g.use_counts();
    for (auto& n : g.nodes) {
      if (n.deleted) continue;
      if (n.op == OP_ADD && n.inputs.size() == 2) {
        for (int side = 0; side < 2 && !changed; ++side) {
          const int32_t gid = n.inputs[side];
          const int32_t oid = n.inputs[1 - side];
          Node& gm = g.node(gid);
          if (gm.deleted || gm.op != OP_GEMM || uc[gid] != 1 || gid == g.output_id) continue;
          if (gid == oid) continue;
          const Shape& os = g.node(oid).shape;
          const int64_t N = gm.shape.dims[gm.shape.rank - 1];
          const bool no_bias = !(gm.epi & (EPI_BIAS_FIRST | EPI_BIAS_LAST));
          Node f = gm;
          if (no_bias && !(gm.epi & (EPI_RELU_PRE | EPI_RESIDUAL)) &&
              (is_bias_vector(os, N) || same_shape(os, gm.shape))) {
            f.bias_id = oid;
            f.epi |= EPI_BIAS_LAST;
            if (!is_bias_vector(os, N)) f.epi |= EPI_BIAS_ROWS;
          } else if (!(gm.epi & (EPI_RESIDUAL | EPI_RELU_POST)) && same_shape(os, gm.shape)) {
            f.residual_id = oid;
            f.epi |= EPI_RESIDUAL;
          } else {
            continue;
          }
          f.inputs.push_back(oid);
          gm.deleted = true;
          become(g, n.id, f);
          changed = true;
        }
        if (changed) break;
      } else if (n.op == OP_RELU && n.inputs.size() == 1) {
        const int32_t gid = n.inputs[0];
        Node& gm = g.node(gid);
        if (gm.deleted || gm.op != OP_GEMM || uc[gid] != 1 || gid == g.output_id) continue;
        Node f = gm;
        if (gm.epi & EPI_RESIDUAL) {
          if (gm.epi & EPI_RELU_POST) continue;
          f.epi |= EPI_RELU_POST;
        } else {
          if (gm.epi & EPI_RELU_PRE) continue;
          f.epi |= EPI_RELU_PRE;
        }
        gm.deleted = true;
        become(g, n.id, f);
        changed = true;
        break;
      }
    }
  }
  for (auto& n : g.nodes) {
    if (n.deleted || n.op != OP_FLATTEN || n.id == g.output_id) continue;
    int32_t src = n.inputs[0];
    while (g.node(src).op == OP_FLATTEN && g.node(src).alias_of >= 0) src = g.node(src).alias_of;
    n.alias_of = src;
  }
}

// ---------------------------------------------------------------------------
// arena plan
// ---------------------------------------------------------------------------
const Alloc* ArenaPlan::find(int32_t id) const {
  for (const auto& a : allocs)
    if (a.node_id == id) return &a;
  return nullptr;
}

static size_t align_up(size_t v, size_t a) {
  if (v > std::numeric_limits<size_t>::max() - (a - 1)) throw std::overflow_error("arena size overflow");
  return ((v + a - 1) / a) * a;
}

ArenaPlan plan_arena(const Graph& g, int64_t max_batch, size_t alignment) {
  if (alignment == 0 || (alignment & (alignment - 1)))
    throw std::invalid_argument("alignment must be a power of two");
  ArenaPlan plan;
  const auto order = g.order();
  std::unordered_map<int32_t, int> step;
  for (size_t s = 0; s < order.size(); ++s) step[order[s]] = static_cast<int>(s);
  // a FLATTEN view extends the life of the buffer it views
  auto owner = [&](int32_t id) {
    while (g.node(id).alias_of >= 0) id = g.node(id).alias_of;
    return id;
  };
  std::unordered_map<int32_t, int> last_use;
  for (int32_t id : order) {
    for (int32_t in : g.node(id).inputs) {
      const int32_t o = owner(in);
      last_use[o] = std::max(last_use[o], step[id]);
    }
  }
  std::vector<Alloc> cands;
  for (int32_t id : order) {
    const Node& n = g.node(id);
    if (n.op == OP_INPUT || n.op == OP_CONST || id == g.output_id || n.alias_of >= 0) continue;
    Alloc a;
    a.node_id = id;
    a.birth = step[id];
    a.death = std::max(a.birth, last_use.count(id) ? last_use[id] : a.birth);
    const int64_t count = n.shape.elems(max_batch);
    if (count < 0 || count > (INT64_MAX / 4)) throw std::overflow_error("tensor too large");
    a.size_bytes = align_up(static_cast<size_t>(count) * sizeof(float), alignment);
    plan.naive_bytes += a.size_bytes;
    cands.push_back(a);
  }
  std::vector<Alloc> placed;
  for (auto& a : cands) {
    auto overlaps = [&](const Alloc& p) { return !(a.death < p.birth || p.death < a.birth); };
    std::vector<size_t> offs{0};
    for (const auto& p : placed)
      if (overlaps(p)) offs.push_back(p.offset + p.size_bytes);
    std::sort(offs.begin(), offs.end());
    offs.erase(std::unique(offs.begin(), offs.end()), offs.end());
    bool found = false;
    size_t best = 0;
    for (size_t c : offs) {
      const size_t ca = align_up(c, alignment);
      bool collide = false;
      for (const auto& p : placed) {
        if (!overlaps(p)) continue;
        if (std::max(ca, p.offset) < std::min(ca + a.size_bytes, p.offset + p.size_bytes)) {
          collide = true;
          break;
        }
      }
      if (!collide) {
        best = ca;
        found = true;
        break;
      }
    }
    if (!found) best = align_up(plan.arena_bytes, alignment);
    a.offset = best;
    placed.push_back(a);
    plan.arena_bytes = std::max(plan.arena_bytes, a.offset + a.size_bytes);
  }
  for (size_t s = 0; s < order.size(); ++s) {
    size_t live = 0;
    for (const auto& a : cands)
      if (a.birth <= static_cast<int>(s) && static_cast<int>(s) <= a.death) live += a.size_bytes;
    plan.peak_live_bytes = std::max(plan.peak_live_bytes, live);
  }
  if (plan.naive_bytes > 0)
    plan.savings_percent = 100.0 * (1.0 - double(plan.arena_bytes) / double(plan.naive_bytes));
  plan.allocs = placed;
  return plan;
}

// ---------------------------------------------------------------------------
// launch list
// ---------------------------------------------------------------------------
static Operand operand_of(const Graph& g, const ArenaPlan& p, int32_t id) {
  while (g.node(id).alias_of >= 0) id = g.node(id).alias_of;
  Operand o;
  const Node& n = g.node(id);
  if (id == g.output_id) {
    o.space = SP_OUTPUT;
  } else if (n.op == OP_INPUT) {
    o.space = SP_INPUT;
  } else if (n.op == OP_CONST) {
    o.space = SP_WEIGHT;
    o.offset = n.const_offset;
  } else {
    const Alloc* a = p.find(id);
    if (!a) throw std::runtime_error("internal: node without arena slot");
    o.space = SP_ARENA;
    o.offset = a->offset;
  }
  return o;
}

static void require(bool c, const std::string& msg) {
  if (!c) throw std::runtime_error(msg);
}

Program build_program(const void* blob, size_t bytes) {
  Program prog;
  prog.graph = parse_blob(blob, bytes);
  Graph& g = prog.graph;
  const bool fusion = (g.flags & BLOB_FUSION) != 0;
  fuse(g, fusion, fusion && !(g.flags & BLOB_NO_FOLD));
  prog.plan = plan_arena(g, g.max_batch, 64);
  const Node& in = g.node(g.input_id);
  const Node& out = g.node(g.output_id);
  prog.dynamic = (g.flags & BLOB_DYNAMIC) != 0 && in.shape.dynamic();
  prog.output_dynamic = out.shape.dynamic();
  prog.in_static_elems = in.shape.static_elems();
  prog.out_static_elems = out.shape.static_elems();
  prog.max_batch = g.max_batch;
  prog.static_batch = in.shape.rank > 0 ? in.shape.dims[0] : 1;
  if (!prog.dynamic) prog.max_batch = prog.static_batch;

  for (int32_t id : g.order()) {
    const Node& n = g.node(id);
    if (n.op == OP_INPUT || n.op == OP_CONST) continue;
    if (n.alias_of >= 0) continue;  // FLATTEN view: no work
    Step s;
    s.node_id = id;
    s.out = operand_of(g, prog.plan, id);
    const bool dyn = n.shape.dynamic();
    s.static_rows = !dyn;
    switch (n.op) {
      case OP_GEMM: {
        const Node& x = g.node(n.inputs[0]);
        const Node& w = g.node(n.inputs[1]);
        require(w.op == OP_CONST && w.shape.rank == 2, "MATMUL: right operand must be a constant [K,N] matrix");
        require(x.shape.rank == 2, "MATMUL: left operand must be rank 2");
        s.kind = ST_GEMM;
        s.K = x.shape.dims[1];
        s.N = w.shape.dims[1];
        require(w.shape.dims[0] == s.K, "MATMUL: inner dimensions differ");
        s.a = operand_of(g, prog.plan, n.inputs[0]);
        s.b = operand_of(g, prog.plan, n.inputs[1]);
        s.epi = n.epi;
        if (n.bias_id >= 0) s.bias = operand_of(g, prog.plan, n.bias_id);
        if (n.residual_id >= 0) s.res = operand_of(g, prog.plan, n.residual_id);
        s.rows_per_sample = dyn ? 1 : x.shape.dims[0];
        break;
      }
      case OP_CONV: {
        const Node& x = g.node(n.inputs[0]);
        const Node& w = g.node(n.inputs[1]);
        require(w.op == OP_CONST && w.shape.rank == 4 && x.shape.rank == 4, "CONV2D: needs NCHW input and OIHW constant weight");
        s.kind = ST_CONV;
        s.Cin = x.shape.dims[1];
        s.H = x.shape.dims[2];
        s.W = x.shape.dims[3];
        s.Cout = w.shape.dims[0];
        require(w.shape.dims[1] == s.Cin, "CONV2D: channel mismatch");
        s.Kh = w.shape.dims[2];
        s.Kw = w.shape.dims[3];
        s.Ho = n.shape.dims[2];
        s.Wo = n.shape.dims[3];
        s.conv = n.conv;
        s.K = s.Cin * s.Kh * s.Kw;
        s.N = s.Cout;
        s.a = operand_of(g, prog.plan, n.inputs[0]);
        s.b = operand_of(g, prog.plan, n.inputs[1]);
        s.epi = n.epi;
        if (n.bias_id >= 0) s.bias = operand_of(g, prog.plan, n.bias_id);
        s.rows_per_sample = dyn ? 1 : x.shape.dims[0];
        break;
      }
      case OP_ADD:
      case OP_MUL: {
        const Node& a = g.node(n.inputs[0]);
        const Node& b = g.node(n.inputs[1]);
        const bool add = n.op == OP_ADD;
        s.a = operand_of(g, prog.plan, n.inputs[0]);
        s.b = operand_of(g, prog.plan, n.inputs[1]);
        s.elems_per_sample = n.shape.static_elems();
        if (same_shape(a.shape, b.shape)) {
          s.kind = add ? ST_ADD_SAME : ST_MUL_SAME;
        } else if (a.shape.rank == 2 && (b.shape.rank == 1 || (b.shape.rank == 2 && b.shape.dims[0] == 1))) {
          s.kind = add ? ST_ADD_ROW : ST_MUL_ROW;
          s.row_len = a.shape.dims[1];
        } else if (a.shape.rank == 4) {
          s.kind = add ? ST_ADD_CHANNEL : ST_MUL_CHANNEL;
          s.channels = a.shape.dims[1];
          s.row_len = a.shape.dims[2] * a.shape.dims[3];
        } else {
          throw std::runtime_error("ADD/MUL: unsupported broadcast");
        }
        break;
      }
      case OP_RELU:
      case OP_SIGMOID:
      case OP_TANH:
      case OP_FLATTEN:
      case OP_OUTPUT: {
        s.kind = n.op == OP_RELU ? ST_RELU : n.op == OP_SIGMOID ? ST_SIGMOID : n.op == OP_TANH ? ST_TANH : ST_COPY;
        s.a = operand_of(g, prog.plan, n.inputs[0]);
        s.elems_per_sample = n.shape.static_elems();
        break;
      }
      default:
        throw std::runtime_error(std::string("unsupported op ") + op_name(n.op));
    }
    prog.steps.push_back(s);
  }
  // identity / constant outputs (src/codegen.cpp:976-993)
  const Node& o = g.node(g.output_id);
  if (o.op == OP_INPUT || o.op == OP_CONST) {
    Step s;
    s.node_id = o.id;
    s.kind = o.op == OP_INPUT ? ST_COPY : ST_FILL_CONST;
    s.out.space = SP_OUTPUT;
    s.a.space = o.op == OP_INPUT ? SP_INPUT : SP_WEIGHT;
    s.a.offset = o.op == OP_CONST ? o.const_offset : 0;
    s.elems_per_sample = o.shape.static_elems();
    s.static_rows = !o.shape.dynamic();
    prog.steps.push_back(s);
  }
  // small-N heads a tensor-core GEMM may compute in its epilogue
  const auto uc = g.use_counts();
  for (size_t i = 0; i + 1 < prog.steps.size(); ++i) {
    Step& a = prog.steps[i];
    Step& b = prog.steps[i + 1];
    if (a.kind != ST_GEMM || b.kind != ST_GEMM || a.static_rows || b.static_rows) continue;
    if (a.out.space != SP_ARENA || b.a.space != SP_ARENA || b.a.offset != a.out.offset) continue;
    if (uc.at(static_cast<size_t>(a.node_id)) != 1) continue;
    if (b.K != a.N || b.N > kMaxHeadN || a.N > kMaxHeadK) continue;
    if (b.epi & (EPI_RESIDUAL | EPI_BIAS_ROWS)) continue;
    if (b.bias.space != SP_NONE && b.bias.space != SP_WEIGHT) continue;
    a.head_step = static_cast<int32_t>(i + 1);
    b.head_of = static_cast<int32_t>(i);
  }
  // two consecutive Linear layers one kernel may compute together
  for (size_t i = 0; i + 1 < prog.steps.size(); ++i) {
    Step& a = prog.steps[i];
    Step& b = prog.steps[i + 1];
    if (a.kind != ST_GEMM || b.kind != ST_GEMM || a.static_rows || b.static_rows) continue;
    if (a.mlp_of >= 0 || a.head_of >= 0) continue;  // a is already absorbed by its predecessor
    if (a.out.space != SP_ARENA || b.a.space != SP_ARENA || b.a.offset != a.out.offset) continue;
    if (uc.at(static_cast<size_t>(a.node_id)) != 1) continue;
    if (b.K != a.N || a.N < kMlpMinN1 || a.N > kMlpMaxN1 || b.N < kMlpMinN2 || b.N > kMlpMaxN2) continue;
    const uint32_t bad = EPI_RESIDUAL | EPI_BIAS_ROWS;
    if ((a.epi & bad) || (b.epi & bad)) continue;
    if (a.bias.space != SP_NONE && a.bias.space != SP_WEIGHT) continue;
    if (b.bias.space != SP_NONE && b.bias.space != SP_WEIGHT) continue;
    if (b.b.space != SP_WEIGHT || a.b.space != SP_WEIGHT) continue;
    a.mlp_step = static_cast<int32_t>(i + 1);
    b.mlp_of = static_cast<int32_t>(i);
  }
  apply_tuning(prog.steps, g.tuning);
  return prog;
}

void apply_tuning(std::vector<Step>& steps, const std::vector<TuneRecord>& records) {
  for (size_t i = 0; i < records.size(); ++i) {
    const TuneRecord& r = records[i];
    std::string why = check_tune_record(r);
    if (why.empty() && (r.step < 0 || r.step >= static_cast<int64_t>(steps.size())))
      why = "step index out of range";
    if (why.empty() && steps[static_cast<size_t>(r.step)].kind != ST_GEMM) why = "step is not a GEMM";
    if (!why.empty()) throw std::runtime_error("tuning record " + std::to_string(i) + ": " + why);
  }
  for (auto& st : steps) st.tuned.clear();
  for (const auto& r : records) steps[static_cast<size_t>(r.step)].tuned.push_back(r);
}

static const char* space_name(int32_t s) {
  switch (s) {
    case SP_INPUT: return "input";
    case SP_OUTPUT: return "output";
    case SP_ARENA: return "arena";
    case SP_WEIGHT: return "weight";
    default: return "none";
  }
}

std::string Program::describe() const {
  std::ostringstream os;
  os << "{\"dynamic\":" << (dynamic ? "true" : "false") << ",\"max_batch\":" << max_batch
     << ",\"static_batch\":" << static_batch << ",\"in_elems\":" << in_static_elems
     << ",\"out_elems\":" << out_static_elems << ",\"arena_bytes\":" << plan.arena_bytes
     << ",\"naive_bytes\":" << plan.naive_bytes << ",\"peak_live_bytes\":" << plan.peak_live_bytes
     << ",\"savings_percent\":" << plan.savings_percent << ",\"allocs\":[";
  for (size_t i = 0; i < plan.allocs.size(); ++i) {
    const auto& a = plan.allocs[i];
    os << (i ? "," : "") << "{\"node\":" << a.node_id << ",\"offset\":" << a.offset
       << ",\"bytes\":" << a.size_bytes << ",\"birth\":" << a.birth << ",\"death\":" << a.death << "}";
  }
  os << "],\"nodes\":[";
  bool first = true;
  for (int32_t id : graph.order()) {
    const Node& n = graph.node(id);
    os << (first ? "" : ",") << "{\"id\":" << id << ",\"op\":\"" << op_name(n.op) << "\",\"epi\":" << n.epi
       << ",\"alias_of\":" << n.alias_of << ",\"inputs\":[";
    for (size_t k = 0; k < n.inputs.size(); ++k) os << (k ? "," : "") << n.inputs[k];
    os << "]}";
    first = false;
  }
  os << "],\"steps\":[";
  for (size_t i = 0; i < steps.size(); ++i) {
    const auto& s = steps[i];
    os << (i ? "," : "") << "{\"kind\":" << s.kind << ",\"node\":" << s.node_id << ",\"K\":" << s.K
       << ",\"N\":" << s.N << ",\"epi\":" << s.epi << ",\"a\":\"" << space_name(s.a.space) << "\",\"out\":\""
       << space_name(s.out.space) << "\",\"out_offset\":" << s.out.offset << ",\"head_step\":" << s.head_step
       << ",\"head_of\":" << s.head_of << ",\"mlp_step\":" << s.mlp_step << ",\"mlp_of\":" << s.mlp_of
       << ",\"tuned\":[";
    for (size_t k = 0; k < s.tuned.size(); ++k) {
      const auto& r = s.tuned[k];
      os << (k ? "," : "") << "[" << r.batch_lo << "," << r.batch_hi << "," << r.family << "," << r.bn << "," << r.bk
         << "," << r.mh << "," << r.pair << "," << (r.fuse_head ? 1 : 0) << "]";
    }
    os << "]}";
  }
  os << "]}";
  return os.str();
}

}  // namespace ftb
