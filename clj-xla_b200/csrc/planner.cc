// Graph -> launch plan.
//
// 1. Dead code is dropped (the printed graphs carry unused RoPE branches:
//    gemma.clj:173,177 compute q- and k-rotations twice).
// 2. Values are classified: splat constants become immediates; reshape /
//    transpose / broadcast_in_dim / slice / identity converts become strided
//    views (no kernel); elementwise ops are grouped into fused register
//    programs; every other op is one kernel.
// 3. Elementwise grouping is cycle safe: a node may join an operand's group
//    only if all the group's external inputs are produced before the group's
//    first member, so the group can run as one kernel.
// 4. Kernel units are ordered topologically (Kahn, earliest member first);
//    views that a consumer cannot read in place are materialised on demand.
// 5. Scratch buffers get arena offsets by liveness over the launch order.
//
// Device pointers go through the argument table (see kernels.h):
//   [params P][outputs O][constant blob 1][scratch buffers T].
#include "planner.h"
#include "fast_kernels.h"

#include <algorithm>
#include <climits>
#include <cmath>
#include <functional>
#include <map>
#include <queue>
#include <set>


namespace cljxla {

const char* kernel_kind_name(int k) {
  static const char* n[] = {"fused_elementwise", "reduce", "copy", "gather", "dynamic_update_slice",
                            "gemm_generic", "gemv", "attention", "attn_combine", "rownorm", "gemm_tc", "fused_multi",
                            "all_reduce", "gemv_fused", "fused_kv_write", "argmax", "gemv_tail"};
  return k >= 0 && k < K_NUM_KINDS ? n[k] : "?";
}

namespace {

// an environment switch set to 0 (for measuring a path against its alternative)
bool getenv_off(const char* name) {
  const char* e = getenv(name);
  return e && e[0] == '0';
}

template <class T>
std::vector<uint8_t> blob_of(const T& p) {
  std::vector<uint8_t> b(sizeof(T));
  memcpy(b.data(), &p, sizeof(T));
  return b;
}

bool is_view_op(const Node& n, const Graph& g) {
  switch (n.op) {
    case Op::Reshape: case Op::Transpose: case Op::Broadcast: case Op::Slice: return true;
    case Op::Convert: return g.nodes[n.in[0]].dt == n.dt;
    default: return false;
  }
}

std::vector<int64_t> dense_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> s(shape.size());
  int64_t acc = 1;
  for (int i = (int)shape.size() - 1; i >= 0; --i) {
    s[i] = acc;
    acc *= shape[i];
  }
  return s;
}

// Strides for `nshape` over memory described by (oshape, ostr), or false if
// the reshape cannot be expressed as a strided view.
bool reshape_strides(const std::vector<int64_t>& oshape, const std::vector<int64_t>& ostr,
                     const std::vector<int64_t>& nshape, std::vector<int64_t>& nstr) {
  std::vector<int64_t> os, ost;
  for (size_t i = 0; i < oshape.size(); ++i)
    if (oshape[i] != 1) { os.push_back(oshape[i]); ost.push_back(ostr[i]); }
  nstr.assign(nshape.size(), 0);
  size_t oi = 0;
  size_t ni = 0;
  while (ni < nshape.size() || oi < os.size()) {
    if (ni < nshape.size() && nshape[ni] == 1) { nstr[ni] = 0; ++ni; continue; }
    if (oi >= os.size() || ni >= nshape.size()) return false;
    // take a chunk of old dims and new dims with equal products
    int64_t op = os[oi], np = nshape[ni];
    size_t oj = oi + 1, nj = ni + 1;
    while (op != np) {
      if (op < np) {
        if (oj >= os.size()) return false;
        op *= os[oj++];
      } else {
        while (nj < nshape.size() && nshape[nj] == 1) nj++;
        if (nj >= nshape.size()) return false;
        np *= nshape[nj++];
      }
    }
    // old dims [oi, oj) must be mutually contiguous
    for (size_t k = oi; k + 1 < oj; ++k)
      if (ost[k] != ost[k + 1] * os[k + 1]) return false;
    int64_t stride = ost[oj - 1];
    for (size_t k = nj; k-- > ni;) {
      if (nshape[k] == 1) { nstr[k] = 0; continue; }
      nstr[k] = stride;
      stride *= nshape[k];
    }
    oi = oj;
    ni = nj;
  }
  return true;
}

int kdt(DT t) { return (int)t; }

// host evaluation of elementwise ops on splat constants (same semantics as the
// device interpreter: f32 arithmetic rounded to the result type; int32 ints)
double round_host(double v, DT dt) {
  switch (dt) {
    case DT::F32: return (double)(float)v;
    case DT::BF16: return (double)bf16_to_f32(f32_to_bf16((float)v));
    case DT::F16: return (double)f16_to_f32(f32_to_f16((float)v));
    case DT::I1: return v != 0 ? 1 : 0;
    default: return (double)(int32_t)(int64_t)v;
  }
}

bool fold_splat(const Node& n, const std::vector<double>& a, const std::vector<DT>& adt, double& out) {
  const bool fl = dt_is_float(n.dt);
  float x = a.size() > 0 ? (float)a[0] : 0.f, y = a.size() > 1 ? (float)a[1] : 0.f;
  double r;
  switch (n.op) {
    case Op::Add: r = fl ? (double)(x + y) : (double)((int32_t)a[0] + (int32_t)a[1]); break;
    case Op::Sub: r = fl ? (double)(x - y) : (double)((int32_t)a[0] - (int32_t)a[1]); break;
    case Op::Mul: r = fl ? (double)(x * y) : (double)((int32_t)a[0] * (int32_t)a[1]); break;
    case Op::Div:
      if (fl) r = (double)(x / y);
      else if ((int32_t)a[1] == 0) return false;
      else r = (double)((int32_t)a[0] / (int32_t)a[1]);
      break;
    case Op::Max: r = fl ? (double)fmaxf(x, y) : std::max(a[0], a[1]); break;
    case Op::Min: r = fl ? (double)fminf(x, y) : std::min(a[0], a[1]); break;
    case Op::Neg: r = fl ? (double)(-x) : -a[0]; break;
    case Op::Sqrt: if (!fl) return false; r = (double)sqrtf(x); break;
    case Op::Convert:
      if (fl) r = dt_is_float(adt[0]) ? (double)(float)a[0] : (double)(float)a[0];
      else if (n.dt == DT::I1) r = a[0] != 0;
      else r = dt_is_float(adt[0]) ? std::trunc(a[0]) : a[0];
      break;
    case Op::Select: r = a[0] != 0 ? a[1] : a[2]; break;
    case Op::Compare: {
      bool c;
      switch (n.i0) {
        case CMP_EQ: c = a[0] == a[1]; break;
        case CMP_NE: c = a[0] != a[1]; break;
        case CMP_GE: c = a[0] >= a[1]; break;
        case CMP_GT: c = a[0] > a[1]; break;
        case CMP_LE: c = a[0] <= a[1]; break;
        default: c = a[0] < a[1]; break;
      }
      r = c;
      break;
    }
    default: return false;  // transcendental splats are left to the device
  }
  out = round_host(r, n.dt);
  return true;
}

struct Loc {
  enum Kind { NONE, SPLAT, BUF, VIEWOP, EW, ROW } kind = NONE;
  double splat = 0;
  int slot = -1;  // argtab slot of the node's buffer (BUF / materialised EW)
};

// A fused row region (see k_row.cu): per-element members over the loop shape
// F, last-axis reductions, per-row scalar members, and the reshape /
// broadcast views connecting them.
struct RowRegion {
  int root = -1;  // first reduce: the unit id
  std::vector<int64_t> F;
  std::set<int> full, scalar, reduces;
  std::map<int, int> alias;  // view node -> member whose value it is (scalar aliases and broadcasts)
  std::set<int> bcast;       // aliases that broadcast a scalar back to F
  std::set<int> all() const {
    std::set<int> s(full);
    s.insert(scalar.begin(), scalar.end());
    s.insert(reduces.begin(), reduces.end());
    for (auto& kv : alias) s.insert(kv.first);
    return s;
  }
};

class Planner {
 public:
  Planner(const Graph& g, const PlanOptions& o, Plan& p) : g_(g), opt_(o), plan_(p) {}
  void run();

 private:
  const Graph& g_;
  PlanOptions opt_;
  Plan& plan_;
  int P_ = 0, O_ = 0, U_ = 0;
  std::map<int, int> inplace_of_;             // dynamic_update_slice node -> index in plan_.inplace
  std::vector<Loc> loc_;
  std::vector<char> live_;
  std::vector<std::vector<int>> users_;
  std::vector<std::vector<int>> ins_;         // operands (fused kernels override the graph's)
  std::map<int, AttnMatch> attn_;             // probs.V dot -> matched attention block
  std::map<int, MaskForm> mask_form_;         // probs.V dot -> its mask, proven a causal / window form
  std::map<int, int> argmax_;                 // final i32 reduce of a printed argmax -> the float logits it reads
  int match_argmax(int r) const;
  std::vector<RowRegion> regions_;
  std::vector<int> region_of_;                // node -> region index or -1
  std::vector<int> uf_;                       // union-find parent (EW nodes)
  std::vector<int> gmin_, gext_, gsize_, gin_;
  std::vector<int> out_claim_;                // node -> output index claimed, or -1
  std::vector<int> mat_slot_;                 // view node -> scratch slot of its materialised copy
  std::vector<int64_t> tmp_bytes_;            // scratch buffer sizes
  std::vector<int> tmp_first_, tmp_last_;     // liveness (launch indices)

  int find(int x) { while (uf_[x] != x) x = uf_[x] = uf_[uf_[x]]; return x; }
  int tmp_slot(int b) const { return P_ + O_ + U_ + 1 + b; }
  int new_tmp(int64_t bytes) {
    tmp_bytes_.push_back(std::max<int64_t>(bytes, 1));
    tmp_first_.push_back((int)plan_.launches.size());
    tmp_last_.push_back((int)plan_.launches.size());
    return tmp_slot((int)tmp_bytes_.size() - 1);
  }
  void touch(int slot) {
    int b = slot - (P_ + O_ + U_ + 1);
    if (b >= 0) tmp_last_[b] = std::max(tmp_last_[b], (int)plan_.launches.size());
  }
  int view_root(int n) const {
    while (is_view_op(g_.nodes[n], g_)) n = g_.nodes[n].in[0];
    return n;
  }
  bool is_splat(int n) const { return loc_[n].kind == Loc::SPLAT; }
  // an elementwise node computed inside the fused concatenates that use it
  // (one op of one memory operand and splats, e.g. the negated half of RoPE's
  // rotate_half): no buffer, no launch of its own
  bool concat_inline(int o) const;
  int concat_inline_operand(int o) const;

  void classify();
  void group_elementwise();
  void decide_materialisation();
  void emit_all();
  void emit_unit(int u);
  void emit_ew_group(const std::vector<int>& members);
  void emit_node_kernel(int n);
  GemmParams dot_params(int id, int oslot, int64_t* bytes, int64_t* flops);
  bool emit_split_dot(int id, int oslot);
  // tile width, A rows per copy and K splits of a tensor-core GEMM (narrow
  // tiles and split K for a few rows of A), with the tensor-map boxes and the
  // split-K partials / counters they need
  void tc_tiling(TcGemmParams& tc, TmapSpec& ta, TmapSpec& tb) {
    int bn = 256, ab = 128, ks = 1;
    if (!getenv_off("CLJXLA_B200_TC_NARROW"))
      tc_gemm_choose(tc.M, tc.N, (int64_t)tc.K * tc.a_parts, 148, &bn, &ab, &ks);
    tc.bn = bn;
    tc.a_box = ab;
    tc.ksplit = ks;
    ta.box_outer = ab;
    tb.box_outer = bn;
    if (ks > 1) {
      tc.part = slot_ptr(new_tmp((int64_t)ks * tc.M * tc.N * 4));
      const int64_t tiles = ((tc.M + 127) / 128) * ((tc.N + bn - 1) / bn);
      const size_t off = (plan_.const_blob.size() + 15) & ~size_t(15);
      plan_.const_blob.resize(off + 4 * tiles, 0);
      tc.counters = slot_ptr(P_ + O_ + U_, (int64_t)off);
    }
  }
  std::set<int> pre_emitted_;  // units already emitted together with an earlier one (grouped GEMVs)
  std::set<int> emitted_units_;
  void build_row_regions();
  void emit_row_region(int r);
  void emit_attention(int d2);
  bool splat_value(int n, double& v);
  void emit_outputs();
  void allocate_arena();

 public:
  // pointer/view helpers (used by fast paths too)
  int ensure_buf(int n);
  TView view_of(int n);
  TView dense_view(int slot, DT dt, const std::vector<int64_t>& shape, int64_t eoff = 0);
  TView materialize(const TView& v, const std::vector<int64_t>& shape, DT dt);
  void push(int kind, std::vector<uint8_t> blob, const std::string& label, int64_t bytes = 0, int64_t flops = 0) {
    Launch l;
    l.kind = kind;
    l.blob = std::move(blob);
    l.label = label;
    l.algo_bytes = bytes;
    l.algo_flops = flops;
    plan_.launches.push_back(std::move(l));
  }
  DPtr slot_ptr(int slot, int64_t off_bytes = 0) {
    DPtr p;
    p.slot = slot;
    p.pad_ = 0;
    p.off = off_bytes;
    touch(slot);
    return p;
  }
};

void Planner::classify() {
  const int N = (int)g_.nodes.size();
  loc_.assign(N, Loc());
  for (int i = 0; i < N; ++i) {
    const Node& n = g_.nodes[i];
    if (!live_[i]) continue;
    if (n.dt == DT::I64 || n.dt == DT::F64)
      fail(E_UNIMPLEMENTED, std::string("element type ") + dt_name(n.dt) + " is not supported on this device path");
    if (n.rank() > CLJXLA_MAXR) fail(E_UNIMPLEMENTED, "rank > 8 is not supported");
    Loc& L = loc_[i];
    if (n.op == Op::Param) { L.kind = Loc::BUF; continue; }
    if (n.op == Op::Constant) {
      if (n.splat) { L.kind = Loc::SPLAT; L.splat = n.splat_val; continue; }
      L.kind = Loc::BUF;
      size_t off = (plan_.const_blob.size() + 255) & ~size_t(255);
      plan_.const_blob.resize(off + n.data.size());
      memcpy(plan_.const_blob.data() + off, n.data.data(), n.data.size());
      L.slot = P_ + O_ + U_;  // const blob; offset recorded in splat field
      L.splat = (double)off;
      continue;
    }
    if (is_view_op(n, g_)) {
      if (is_splat(n.in[0])) {
        L.kind = Loc::SPLAT;
        L.splat = loc_[n.in[0]].splat;
      } else {
        L.kind = Loc::VIEWOP;
      }
      continue;
    }
    if (op_is_elementwise(n.op)) {
      bool all_splat = n.op != Op::Iota;
      std::vector<double> a;
      std::vector<DT> adt;
      for (int x : n.in) {
        all_splat &= is_splat(x);
        a.push_back(loc_[x].splat);
        adt.push_back(g_.nodes[x].dt);
      }
      double v;
      if (all_splat && !n.in.empty() && fold_splat(n, a, adt, v)) {
        L.kind = Loc::SPLAT;
        L.splat = v;
        continue;
      }
      L.kind = Loc::EW;
      continue;
    }
    if (n.op == Op::Concat && opt_.fuse) {
      bool ok = true;
      for (int x : n.in) ok &= !is_splat(x) && g_.nodes[x].dt == n.dt;
      if (ok) {
        L.kind = Loc::EW;  // fused as range-predicated loads
        continue;
      }
    }
    L.kind = Loc::BUF;  // produced by its own kernel
  }
}

int Planner::concat_inline_operand(int o) const {
  const Node& n = g_.nodes[o];
  int x = -1, cnt = 0;
  for (int i : n.in)
    if (!is_splat(i)) {
      x = i;
      ++cnt;
    }
  return cnt == 1 ? x : -1;
}

bool Planner::concat_inline(int o) const {
  if (!opt_.fuse || !live_[o] || loc_[o].kind != Loc::EW || out_claim_[o] >= 0) return false;
  for (int x : g_.outputs)
    if (x == o) return false;
  const Node& n = g_.nodes[o];
  switch (n.op) {
    case Op::Neg: case Op::Convert:
      if (n.in.size() != 1) return false;
      break;
    case Op::Add: case Op::Sub: case Op::Mul: case Op::Div: case Op::Max: case Op::Min:
      if (n.in.size() != 2) return false;
      break;
    default: return false;
  }
  const int x = concat_inline_operand(o);
  if (x < 0) return false;
  const Loc::Kind xk = loc_[x].kind;
  if (!(xk == Loc::BUF || xk == Loc::VIEWOP || xk == Loc::ROW)) return false;  // read from memory
  for (int u : users_[o])
    if (live_[u] && !(g_.nodes[u].op == Op::Concat && loc_[u].kind == Loc::EW)) return false;
  return true;
}

void Planner::group_elementwise() {
  const int N = (int)g_.nodes.size();
  uf_.resize(N);
  gmin_.assign(N, 0);
  gext_.assign(N, -1);
  gsize_.assign(N, 1);
  gin_.assign(N, 0);
  for (int i = 0; i < N; ++i) uf_[i] = i;
  // groups: members and external (non-splat) operands, keyed by root
  std::map<int, std::vector<int>> members, exts;
  std::vector<int> stamp(N, 0);
  int cur_stamp = 0;
  // true if any external operand can reach a member through the graph
  auto has_path_back = [&](const std::set<int>& mem, const std::set<int>& ext) {
    int lo = *mem.begin();
    ++cur_stamp;
    std::vector<int> stack;
    for (int o : ext) stack.push_back(o);
    while (!stack.empty()) {
      int x = stack.back();
      stack.pop_back();
      if (x < lo || stamp[x] == cur_stamp) continue;
      stamp[x] = cur_stamp;
      if (mem.count(x)) return true;
      for (int y : ins_[x]) stack.push_back(y);
    }
    return false;
  };
  auto inside = [&](int o, const Node& n, const std::set<int>& roots) {
    return loc_[o].kind == Loc::EW && g_.nodes[o].shape == n.shape && roots.count(find(o));
  };
  for (int i = 0; i < N; ++i) {
    if (!live_[i] || loc_[i].kind != Loc::EW) continue;
    const Node& n = g_.nodes[i];
    std::vector<int> cands;
    if (opt_.fuse && n.op != Op::Concat)
      for (int o : n.in)
        if (loc_[o].kind == Loc::EW && g_.nodes[o].shape == n.shape) cands.push_back(find(o));
    std::sort(cands.begin(), cands.end());
    cands.erase(std::unique(cands.begin(), cands.end()), cands.end());
    // candidate merged group: members + external operands, validity test
    auto build = [&](const std::set<int>& roots, std::set<int>& mem, std::set<int>& ext) {
      mem = {i};
      ext.clear();
      for (int G : roots)
        for (int m : members[G]) mem.insert(m);
      for (int G : roots)
        for (int o : exts[G])
          if (!mem.count(o)) ext.insert(o);
      for (int o : n.in)
        if (!is_splat(o) && !inside(o, n, roots)) ext.insert(o);
    };
    auto valid = [&](const std::set<int>& roots) {
      std::set<int> mem, ext;
      build(roots, mem, ext);
      if ((int)mem.size() > 24 || (int)ext.size() > EW_MAXIN - 2) return false;
      for (int x : mem)  // a fused concatenate reads its operands from memory
        if (g_.nodes[x].op == Op::Concat)
          for (int o : g_.nodes[x].in)
            if (mem.count(o)) return false;
      return !has_path_back(mem, ext);
    };
    std::set<int> merged;
    std::set<int> all(cands.begin(), cands.end());
    if (!all.empty() && valid(all)) {
      merged = all;
    } else {
      for (int G : cands) {
        std::set<int> trial = merged;
        trial.insert(G);
        if (valid(trial)) merged = trial;
      }
    }
    std::set<int> mem, ext;
    build(merged, mem, ext);
    for (int M : merged) {
      uf_[M] = i;
      members.erase(M);
      exts.erase(M);
    }
    members[i] = std::vector<int>(mem.begin(), mem.end());
    exts[i] = std::vector<int>(ext.begin(), ext.end());
  }
}

void Planner::decide_materialisation() {
  const int N = (int)g_.nodes.size();
  for (int i = 0; i < N; ++i) {
    if (!live_[i] || loc_[i].kind != Loc::EW) continue;
    if (concat_inline(i)) continue;  // recomputed by the concatenates reading it
    bool need = out_claim_[i] >= 0;
    for (int u : users_[i]) {
      if (!live_[u]) continue;
      bool same = loc_[u].kind == Loc::EW && find(u) == find(i) && g_.nodes[u].shape == g_.nodes[i].shape &&
                  g_.nodes[u].op != Op::Concat;  // a fused concatenate loads its operands
      if (!same) need = true;
    }
    for (int o : g_.outputs) if (o == i) need = true;
    if (need) ensure_buf(i);
  }
}

int Planner::ensure_buf(int n) {
  Loc& L = loc_[n];
  if (L.slot >= 0) return L.slot;
  const Node& nd = g_.nodes[n];
  if (nd.op == Op::Param) {
    for (int k = 0; k < P_; ++k)
      if (g_.params[k] == n) return L.slot = k;
  }
  if (out_claim_[n] >= 0) return L.slot = P_ + out_claim_[n];
  return L.slot = new_tmp(nd.numel() * (int64_t)dt_size(nd.dt));
}

TView Planner::dense_view(int slot, DT dt, const std::vector<int64_t>& shape, int64_t eoff) {
  TView v{};
  v.p = slot_ptr(slot, eoff * (int64_t)dt_size(dt));
  v.dt = kdt(dt);
  v.rank = (int)shape.size();
  auto st = dense_strides(shape);
  for (int i = 0; i < v.rank; ++i) { v.shape[i] = shape[i]; v.stride[i] = st[i]; }
  return v;
}

TView Planner::materialize(const TView& src, const std::vector<int64_t>& shape, DT dt) {
  int slot = new_tmp(numel(shape) * (int64_t)dt_size(dt));
  CopyParams cp{};
  cp.src = src;
  cp.dst = dense_view(slot, dt, shape);
  cp.n = numel(shape);
  push(K_COPY, blob_of(cp), "materialize", 2 * cp.n * (int64_t)dt_size(dt));
  return dense_view(slot, dt, shape);
}

TView Planner::view_of(int n) {
  const Node& nd = g_.nodes[n];
  Loc& L = loc_[n];
  if (L.kind == Loc::SPLAT) fail(E_INTERNAL, "view_of on a splat constant");
  if (L.kind == Loc::BUF && nd.op == Op::Constant) {
    TView v = dense_view(L.slot, nd.dt, nd.shape);
    v.p.off = (int64_t)L.splat;
    return v;
  }
  if (L.kind == Loc::BUF || L.kind == Loc::EW || L.kind == Loc::ROW) {
    if (L.slot < 0 && nd.op == Op::Param) ensure_buf(n);
    if (L.slot < 0) fail(E_INTERNAL, std::string("value %") + nd.name + " is not materialised");
    return dense_view(L.slot, nd.dt, nd.shape);
  }
  // view ops
  if (mat_slot_[n] >= 0) return dense_view(mat_slot_[n], nd.dt, nd.shape);
  if (nd.op == Op::Reshape) {
    // a reshape of a reshape is one reshape of the first one's operand: a
    // head merge followed by the split back (printed around the attention
    // block) stays a strided view instead of a materialised copy
    int src = nd.in[0];
    while (g_.nodes[src].op == Op::Reshape && loc_[src].kind == Loc::VIEWOP && mat_slot_[src] < 0)
      src = g_.nodes[src].in[0];
    if (src != nd.in[0] && g_.nodes[src].dt == nd.dt) {
      TView base = view_of(src);
      std::vector<int64_t> os(base.shape, base.shape + base.rank), ost(base.stride, base.stride + base.rank), ns;
      if (reshape_strides(os, ost, nd.shape, ns)) {
        TView v = base;
        v.rank = nd.rank();
        for (int i = 0; i < v.rank; ++i) v.shape[i] = nd.shape[i], v.stride[i] = ns[i];
        return v;
      }
    }
  }
  TView in = view_of(nd.in[0]);
  TView v = in;
  v.rank = nd.rank();
  for (int i = 0; i < v.rank; ++i) v.shape[i] = nd.shape[i];
  switch (nd.op) {
    case Op::Convert:
      v.dt = kdt(nd.dt);
      break;
    case Op::Transpose:
      for (int i = 0; i < v.rank; ++i) v.stride[i] = in.stride[nd.ia[i]];
      break;
    case Op::Broadcast: {
      for (int i = 0; i < v.rank; ++i) v.stride[i] = 0;
      for (int i = 0; i < in.rank; ++i) {
        int od = (int)nd.ia[i];
        v.stride[od] = (in.shape[i] == nd.shape[od]) ? in.stride[i] : 0;
      }
      break;
    }
    case Op::Slice: {
      int64_t eoff = 0;
      for (int i = 0; i < in.rank; ++i) {
        eoff += nd.ia[i] * in.stride[i];
        v.stride[i] = in.stride[i] * nd.ic[i];
      }
      v.p.off += eoff * (int64_t)dt_size(nd.dt);
      break;
    }
    case Op::Reshape: {
      std::vector<int64_t> os(in.shape, in.shape + in.rank), ost(in.stride, in.stride + in.rank), ns;
      if (reshape_strides(os, ost, nd.shape, ns)) {
        for (int i = 0; i < v.rank; ++i) v.stride[i] = ns[i];
      } else {
        std::vector<int64_t> ishape(in.shape, in.shape + in.rank);
        TView m = materialize(in, ishape, g_.nodes[nd.in[0]].dt);
        mat_slot_[n] = m.p.slot;
        return dense_view(m.p.slot, nd.dt, nd.shape);
      }
      break;
    }
    default: fail(E_INTERNAL, "bad view op");
  }
  return v;
}

void Planner::emit_ew_group(const std::vector<int>& members) {
  EwParams P{};
  const Node& first = g_.nodes[members[0]];
  P.rank = first.rank();
  P.n = first.numel();
  for (int i = 0; i < P.rank; ++i) P.dims[i] = first.shape[i];
  std::map<int, int> reg_of;  // node -> register
  std::map<std::pair<int, int64_t>, int> imm_reg;
  std::map<int, int> load_reg;
  std::set<int> member_set(members.begin(), members.end());
  // last in-group use of each member (for register reuse)
  std::map<int, int> last_use;
  for (size_t k = 0; k < members.size(); ++k)
    for (int o : g_.nodes[members[k]].in)
      if (member_set.count(o)) last_use[o] = (int)k;
  std::vector<int> free_regs;
  for (int r = EW_NREG - 1; r >= 0; --r) free_regs.push_back(r);
  auto alloc_reg = [&]() {
    if (free_regs.empty()) fail(E_INTERNAL, "fused elementwise program needs too many registers");
    int r = free_regs.back();
    free_regs.pop_back();
    return r;
  };
  auto emit = [&](const EwInstr& I) {
    if (P.ncode >= EW_MAXCODE) fail(E_INTERNAL, "fused elementwise program too long");
    P.code[P.ncode++] = I;
  };
  std::vector<std::pair<int, int>> outs;  // (node, reg)
  std::string label;
  int64_t bytes = 0;
  for (size_t k = 0; k < members.size(); ++k) {
    int id = members[k];
    const Node& n = g_.nodes[id];
    if (n.op == Op::Concat) {
      // concatenate: one range-predicated load per (materialised) operand,
      // chained so each loop index takes the operand that covers it
      EwInstr Z{};
      Z.op = EW_IMM;
      Z.dt = (uint8_t)kdt(n.dt);
      Z.dst = (uint8_t)alloc_reg();
      emit(Z);
      int cur = Z.dst;
      int64_t off = 0;
      const int dim = (int)n.i0;
      for (int o : n.in) {
        if (P.nin >= EW_MAXIN) fail(E_INTERNAL, "fused elementwise region has too many inputs");
        const Node& on = g_.nodes[o];
        if (loc_[o].slot < 0 && concat_inline(o)) {
          // computed here: load its memory operand over this operand's index range,
          // apply the op, and keep the result only inside the range
          const int x = concat_inline_operand(o);
          const Node& xn = g_.nodes[x];
          TView v = view_of(x);
          EwIn& in = P.in[P.nin];
          in.p = v.p;
          in.dt = v.dt;
          in.sel_dim = dim;
          in.sel_lo = off;
          in.sel_hi = off + on.shape[dim];
          for (int d = 0; d < P.rank; ++d) in.stride[d] = v.stride[d];
          bytes += xn.numel() * (int64_t)dt_size(xn.dt);
          auto imm = [&](uint8_t dt, double val) {
            EwInstr I{};
            I.op = EW_IMM;
            I.dt = dt;
            I.dst = (uint8_t)alloc_reg();
            I.fimm = (float)val;
            I.iimm = (int32_t)(int64_t)val;
            emit(I);
            return (int)I.dst;
          };
          const int zero = imm((uint8_t)v.dt, 0.0);
          EwInstr L{};
          L.op = EW_LOAD;
          L.dt = (uint8_t)v.dt;
          L.aux = (uint8_t)P.nin;
          L.b = (uint8_t)zero;
          L.dst = (uint8_t)alloc_reg();
          emit(L);
          P.nin++;
          std::vector<int> regs, tmp = {zero};
          for (int i : on.in) {
            if (i == x) {
              regs.push_back(L.dst);
            } else {
              const int r = imm((uint8_t)kdt(g_.nodes[i].dt), loc_[i].splat);
              regs.push_back(r);
              tmp.push_back(r);
            }
          }
          EwInstr I{};
          I.dt = (uint8_t)kdt(on.dt);
          switch (on.op) {
            case Op::Neg: I.op = EW_NEG; break;
            case Op::Convert: I.op = EW_CONVERT; I.aux = (uint8_t)kdt(xn.dt); break;
            case Op::Add: I.op = EW_ADD; break;
            case Op::Sub: I.op = EW_SUB; break;
            case Op::Mul: I.op = EW_MUL; break;
            case Op::Div: I.op = EW_DIV; break;
            case Op::Max: I.op = EW_MAX; break;
            default: I.op = EW_MIN; break;
          }
          I.a = (uint8_t)regs[0];
          I.b = (uint8_t)(regs.size() > 1 ? regs[1] : 0);
          I.dst = (uint8_t)alloc_reg();
          emit(I);
          // index along the concatenated dim within [off, off + len)?
          EwInstr Io{};
          Io.op = EW_IOTA;
          Io.dt = (uint8_t)kdt(DT::I32);
          Io.aux = (uint8_t)dim;
          Io.dst = (uint8_t)alloc_reg();
          emit(Io);
          const int lo = imm((uint8_t)kdt(DT::I32), (double)off);
          const int hi = imm((uint8_t)kdt(DT::I32), (double)(off + on.shape[dim]));
          EwInstr C1{}, C2{}, S1{}, S2{};
          C1.op = C2.op = EW_CMP;
          C1.dt = C2.dt = (uint8_t)kdt(DT::I1);
          C1.aux2 = C2.aux2 = (uint8_t)kdt(DT::I32);
          C1.aux = 2;  // >=
          C1.a = Io.dst;
          C1.b = (uint8_t)lo;
          C1.dst = (uint8_t)alloc_reg();
          emit(C1);
          C2.aux = 5;  // <
          C2.a = Io.dst;
          C2.b = (uint8_t)hi;
          C2.dst = (uint8_t)alloc_reg();
          emit(C2);
          S1.op = S2.op = EW_SELECT;
          S1.dt = S2.dt = (uint8_t)kdt(n.dt);
          S1.a = C1.dst;
          S1.b = I.dst;
          S1.c = (uint8_t)cur;
          S1.dst = (uint8_t)alloc_reg();
          emit(S1);
          S2.a = C2.dst;
          S2.b = S1.dst;
          S2.c = (uint8_t)cur;
          S2.dst = (uint8_t)alloc_reg();
          emit(S2);
          for (int r : tmp) free_regs.push_back(r);
          for (int r : {(int)L.dst, (int)I.dst, (int)Io.dst, lo, hi, (int)C1.dst, (int)C2.dst, (int)S1.dst, cur})
            free_regs.push_back(r);
          cur = S2.dst;
          off += on.shape[dim];
          continue;
        }
        TView v = view_of(o);
        EwIn& in = P.in[P.nin];
        in.p = v.p;
        in.dt = v.dt;
        in.sel_dim = dim;
        in.sel_lo = off;
        in.sel_hi = off + on.shape[dim];
        for (int d = 0; d < P.rank; ++d) in.stride[d] = v.stride[d];
        bytes += on.numel() * (int64_t)dt_size(on.dt);
        EwInstr L{};
        L.op = EW_LOAD;
        L.dt = (uint8_t)v.dt;
        L.aux = (uint8_t)P.nin;
        L.b = (uint8_t)cur;
        L.dst = (uint8_t)alloc_reg();
        emit(L);
        free_regs.push_back(cur);
        cur = L.dst;
        P.nin++;
        off += on.shape[dim];
      }
      reg_of[id] = cur;
      if (loc_[id].slot >= 0) outs.emplace_back(id, cur);
      if (!label.empty()) label += ",";
      if (label.size() < 80) label += n.name;
      continue;
    }
    std::vector<int> regs;
    for (int o : n.in) {
      if (member_set.count(o) && reg_of.count(o)) { regs.push_back(reg_of[o]); continue; }
      const Node& on = g_.nodes[o];
      if (is_splat(o)) {
        double v = loc_[o].splat;
        int64_t key;
        memcpy(&key, &v, 8);
        auto kk = std::make_pair((int)on.dt, key);
        if (!imm_reg.count(kk)) {
          EwInstr I{};
          I.op = EW_IMM;
          I.dt = (uint8_t)kdt(on.dt);
          I.dst = (uint8_t)alloc_reg();
          I.fimm = (float)v;
          I.iimm = (int32_t)(int64_t)v;
          emit(I);
          imm_reg[kk] = I.dst;
        }
        regs.push_back(imm_reg[kk]);
        continue;
      }
      if (!load_reg.count(o)) {
        if (P.nin >= EW_MAXIN) fail(E_INTERNAL, "fused elementwise region has too many inputs");
        TView v = view_of(o);
        EwIn& in = P.in[P.nin];
        in.p = v.p;
        in.dt = v.dt;
        in.sel_dim = -1;
        for (int d = 0; d < P.rank; ++d) in.stride[d] = v.stride[d];
        bytes += on.numel() * (int64_t)dt_size(on.dt);
        EwInstr I{};
        I.op = EW_LOAD;
        I.dt = (uint8_t)v.dt;
        I.dst = (uint8_t)alloc_reg();
        I.aux = (uint8_t)P.nin;
        emit(I);
        load_reg[o] = I.dst;
        P.nin++;
      }
      regs.push_back(load_reg[o]);
    }
    EwInstr I{};
    I.dt = (uint8_t)kdt(n.dt);
    switch (n.op) {
      case Op::Add: I.op = EW_ADD; break;
      case Op::Sub: I.op = EW_SUB; break;
      case Op::Mul: I.op = EW_MUL; break;
      case Op::Div: I.op = EW_DIV; break;
      case Op::Max: I.op = EW_MAX; break;
      case Op::Min: I.op = EW_MIN; break;
      case Op::Exp: I.op = EW_EXP; break;
      case Op::Tanh: I.op = EW_TANH; break;
      case Op::Sqrt: I.op = EW_SQRT; break;
      case Op::Rsqrt: I.op = EW_RSQRT; break;
      case Op::Sin: I.op = EW_SIN; break;
      case Op::Cos: I.op = EW_COS; break;
      case Op::Logistic: I.op = EW_LOGISTIC; break;
      case Op::Neg: I.op = EW_NEG; break;
      case Op::Abs: I.op = EW_ABS; break;
      case Op::Convert: I.op = EW_CONVERT; I.aux = (uint8_t)kdt(g_.nodes[n.in[0]].dt); break;
      case Op::Compare: I.op = EW_CMP; I.aux = (uint8_t)n.i0; I.aux2 = (uint8_t)kdt(g_.nodes[n.in[0]].dt); break;
      case Op::Select: I.op = EW_SELECT; break;
      case Op::Iota: I.op = EW_IOTA; I.aux = (uint8_t)n.i0; break;
      default: fail(E_INTERNAL, "not an elementwise op");
    }
    if (regs.size() > 0) I.a = (uint8_t)regs[0];
    if (regs.size() > 1) I.b = (uint8_t)regs[1];
    if (regs.size() > 2) I.c = (uint8_t)regs[2];
    // free operand registers whose last use is this instruction (members only)
    for (int o : n.in)
      if (member_set.count(o) && last_use[o] == (int)k && reg_of.count(o) && loc_[o].slot < 0) {
        free_regs.push_back(reg_of[o]);
        reg_of.erase(o);
      }
    I.dst = (uint8_t)alloc_reg();
    emit(I);
    reg_of[id] = I.dst;
    if (loc_[id].slot >= 0) outs.emplace_back(id, I.dst);
    if (!label.empty()) label += ",";
    if (label.size() < 80) label += n.name;
  }
  // collapse the loop shape: drop size-1 dims and merge adjacent dims that are
  // contiguous for every input (outputs are dense), unless an iota needs them
  bool has_iota = false;
  for (int k = 0; k < P.ncode; ++k) has_iota |= P.code[k].op == EW_IOTA;
  for (int i = 0; i < P.nin; ++i) has_iota |= P.in[i].sel_dim >= 0;
  if (!has_iota && P.rank > 1) {
    std::vector<int64_t> dims;
    std::vector<std::vector<int64_t>> st(P.nin);
    for (int d = 0; d < P.rank; ++d) {
      if (P.dims[d] == 1) continue;
      bool merge = !dims.empty();
      for (int i = 0; i < P.nin && merge; ++i) merge = st[i].back() == P.in[i].stride[d] * P.dims[d];
      if (merge) {
        dims.back() *= P.dims[d];
        for (int i = 0; i < P.nin; ++i) st[i].back() = P.in[i].stride[d];
      } else {
        dims.push_back(P.dims[d]);
        for (int i = 0; i < P.nin; ++i) st[i].push_back(P.in[i].stride[d]);
      }
    }
    if (dims.empty()) {
      dims.push_back(1);
      for (int i = 0; i < P.nin; ++i) st[i].push_back(0);
    }
    P.rank = (int)dims.size();
    for (int d = 0; d < CLJXLA_MAXR; ++d) P.dims[d] = d < P.rank ? dims[d] : 0;
    for (int i = 0; i < P.nin; ++i)
      for (int d = 0; d < CLJXLA_MAXR; ++d) P.in[i].stride[d] = d < P.rank ? st[i][d] : 0;
  }
  // outputs, at most EW_MAXOUT per launch (re-run the program for extra chunks)
  for (size_t s = 0; s < outs.size(); s += EW_MAXOUT) {
    EwParams Q = P;
    Q.nout = 0;
    int64_t ob = 0;
    for (size_t k = s; k < outs.size() && Q.nout < EW_MAXOUT; ++k) {
      int id = outs[k].first;
      const Node& n = g_.nodes[id];
      Q.out[Q.nout].p = slot_ptr(loc_[id].slot);
      Q.out[Q.nout].dt = kdt(n.dt);
      Q.out[Q.nout].reg = outs[k].second;
      ob += n.numel() * (int64_t)dt_size(n.dt);
      Q.nout++;
    }
    push(K_EW, blob_of(Q), label, bytes + ob);
  }
}

void Planner::build_row_regions() {
  const int N = (int)g_.nodes.size();
  region_of_.assign(N, -1);
  if (!opt_.fuse) return;
  std::vector<int> stamp(N, 0);
  int cur = 0;
  for (int r0 = 0; r0 < N; ++r0) {
    const Node& R0 = g_.nodes[r0];
    if (!live_[r0] || R0.op != Op::Reduce || region_of_[r0] >= 0 || loc_[r0].kind != Loc::BUF) continue;
    const Node& X = g_.nodes[R0.in[0]];
    if (!dt_is_float(X.dt) || !dt_is_float(R0.dt) || X.rank() < 1 || X.rank() > CLJXLA_MAXR) continue;
    if (R0.ia.size() != 1 || R0.ia[0] != X.rank() - 1 || !is_splat(R0.in[1])) continue;
    RowRegion rg;
    rg.root = r0;
    rg.F = X.shape;
    std::vector<int64_t> sshape(rg.F.begin(), rg.F.end() - 1), sshape1 = sshape;
    sshape1.push_back(1);
    auto in_region = [&](int x) { return rg.full.count(x) || rg.scalar.count(x) || rg.reduces.count(x) || rg.alias.count(x); };
    auto members_min = [&]() {
      int lo = INT32_MAX;
      for (int x : rg.full) lo = std::min(lo, x);
      for (int x : rg.scalar) lo = std::min(lo, x);
      for (int x : rg.reduces) lo = std::min(lo, x);
      return lo;
    };
    // an external operand must not depend on any region member
    auto external_ok = [&](int o) {
      if (is_splat(o)) return true;
      int lo = members_min();
      ++cur;
      std::vector<int> st{o};
      while (!st.empty()) {
        int x = st.back();
        st.pop_back();
        if (x < lo || stamp[x] == cur) continue;
        stamp[x] = cur;
        if (in_region(x)) return false;
        for (int y : ins_[x]) st.push_back(y);
      }
      return true;
    };
    auto is_scalar_val = [&](int o) {  // scalar member / reduce / scalar alias
      if (rg.scalar.count(o) || rg.reduces.count(o)) return true;
      return rg.alias.count(o) && !rg.bcast.count(o);
    };
    auto is_full_val = [&](int o) { return rg.full.count(o) || rg.bcast.count(o); };
    // producers of the reduced value: elementwise nodes of shape F feeding it
    std::vector<int> st{R0.in[0]};
    while (!st.empty()) {
      int x = st.back();
      st.pop_back();
      if (rg.full.count(x)) continue;
      const Node& xn = g_.nodes[x];
      if (loc_[x].kind != Loc::EW || xn.op == Op::Concat || xn.shape != rg.F || region_of_[x] >= 0) continue;
      if (rg.full.size() >= 16) break;
      rg.full.insert(x);
      for (int o : ins_[x]) st.push_back(o);
    }
    rg.reduces.insert(r0);
    // all non-member operands of the producers must be external and independent
    bool ok = true;
    for (int x : rg.full)
      for (int o : ins_[x])
        if (!in_region(o)) ok &= external_ok(o);
    if (!ok) continue;
    // grow forward
    bool changed = true;
    int nphase_red = 1;
    while (changed) {
      changed = false;
      std::set<int> frontier;
      for (int x : rg.all())
        for (int u : users_[x])
          if (live_[u] && !in_region(u) && region_of_[u] < 0) frontier.insert(u);
      for (int u : frontier) {
        const Node& un = g_.nodes[u];
        if ((int)(rg.full.size() + rg.scalar.size()) >= 40) break;
        // scalar aliases: reshape / identity views between [rows] and [rows, 1]
        if (is_view_op(un, g_) && un.op != Op::Broadcast && is_scalar_val(un.in[0]) &&
            (un.shape == sshape || un.shape == sshape1)) {
          rg.alias[u] = un.in[0];
          changed = true;
          continue;
        }
        // broadcast of a per-row scalar back over F (trailing axis broadcast)
        if (un.op == Op::Broadcast && is_scalar_val(un.in[0]) && un.shape == rg.F) {
          const Node& sn = g_.nodes[un.in[0]];
          bool okb = (int)un.ia.size() == sn.rank();
          for (int i = 0; i < (int)un.ia.size() && okb; ++i) okb = un.ia[i] == i;
          if (okb && sn.rank() == (int)rg.F.size() && sn.shape.back() != 1) okb = false;
          if (okb) {
            rg.alias[u] = un.in[0];
            rg.bcast.insert(u);
            changed = true;
          }
          continue;
        }
        if (loc_[u].kind == Loc::EW && un.op != Op::Concat && un.op != Op::Iota) {
          bool all_scalar = true, all_full = true;
          std::vector<int> exts;
          for (int o : ins_[u]) {
            if (is_splat(o)) continue;
            if (!is_scalar_val(o)) all_scalar = false;
            if (!is_full_val(o)) {
              all_full = false;
              exts.push_back(o);
            }
          }
          if ((un.shape == sshape || un.shape == sshape1) && all_scalar &&
              (int)(rg.scalar.size() + rg.reduces.size()) < RP_NREG - RP_SREG0) {
            rg.scalar.insert(u);
            changed = true;
            continue;
          }
          if (un.shape == rg.F) {
            bool ext_ok = true;
            for (int o : exts) ext_ok &= !is_scalar_val(o) && external_ok(o);
            // an external operand must be readable with F-shaped strides
            for (int o : exts) ext_ok &= g_.nodes[o].shape == rg.F;
            if (ext_ok) {
              rg.full.insert(u);
              changed = true;
              // external elementwise operands computed only from values outside
              // the region (the printer's per-consumer converts of a GEMV result)
              // are recomputed inside it instead of costing a launch of their own
              std::vector<int> work(exts.begin(), exts.end());
              while (!work.empty() && (int)(rg.full.size() + rg.scalar.size()) < 40) {
                int o = work.back();
                work.pop_back();
                const Node& on = g_.nodes[o];
                if (rg.full.count(o) || region_of_[o] >= 0 || loc_[o].kind != Loc::EW || on.op == Op::Concat ||
                    on.op == Op::Iota || on.shape != rg.F || !external_ok(o))
                  continue;
                rg.full.insert(o);
                for (int oi : ins_[o])
                  if (!is_splat(oi)) work.push_back(oi);
              }
            }
            (void)all_full;
            continue;
          }
          continue;
        }
        if (un.op == Op::Reduce && loc_[u].kind == Loc::BUF && rg.full.count(un.in[0]) && nphase_red < RP_MAXPH - 1 &&
            un.ia.size() == 1 && un.ia[0] == (int64_t)rg.F.size() - 1 && is_splat(un.in[1]) && dt_is_float(un.dt)) {
          rg.reduces.insert(u);
          nphase_red++;
          changed = true;
        }
      }
    }
    // a region stores at most RP_MAXOUT values; with more (a graph that returns
    // its intermediates) the members stay separate kernels
    std::function<bool(int)> needed = [&](int x) {
      for (int o : g_.outputs)
        if (o == x) return true;
      for (int u : users_[x]) {
        if (!live_[u]) continue;
        if (!in_region(u)) return true;
        if (rg.alias.count(u) && needed(u)) return true;
      }
      return false;
    };
    int nout = 0;
    for (int x : rg.full) nout += needed(x);
    for (int x : rg.scalar) nout += needed(x);
    for (int x : rg.reduces) nout += needed(x);
    if (nout > RP_MAXOUT) continue;
    int id = (int)regions_.size();
    for (int x : rg.all()) region_of_[x] = id;
    for (int x : rg.full) loc_[x].kind = Loc::ROW;
    for (int x : rg.scalar) loc_[x].kind = Loc::ROW;
    for (int x : rg.reduces) loc_[x].kind = Loc::ROW;
    regions_.push_back(std::move(rg));
  }
}

void Planner::emit_row_region(int rid) {
  const RowRegion& rg = regions_[rid];
  RowParams P{};
  P.rank = (int)rg.F.size();
  for (int d = 0; d < P.rank; ++d) P.dims[d] = rg.F[d];
  P.C = rg.F.back();
  P.rows = 1;
  for (int d = 0; d + 1 < P.rank; ++d) P.rows *= rg.F[d];
  auto base = [&](int x) {  // resolve aliases to the member holding the value
    while (rg.alias.count(x)) x = rg.alias.at(x);
    return x;
  };
  // phases
  std::map<int, int> phase, level;
  std::vector<int> order;  // members in index order
  for (int x : rg.full) order.push_back(x);
  for (int x : rg.scalar) order.push_back(x);
  for (int x : rg.reduces) order.push_back(x);
  std::sort(order.begin(), order.end());
  for (int x : order) {
    const Node& n = g_.nodes[x];
    if (rg.full.count(x)) {
      int p = 0;
      for (int o : n.in) {
        if (is_splat(o)) continue;
        int b = base(o);
        if (rg.full.count(b)) p = std::max(p, phase[b]);
        else if (rg.scalar.count(b) || rg.reduces.count(b)) p = std::max(p, level[b]);
      }
      phase[x] = p;
    } else if (rg.reduces.count(x)) {
      phase[x] = phase[n.in[0]];
      level[x] = phase[x] + 1;
    } else {
      int l = 0;
      for (int o : n.in) {
        if (is_splat(o)) continue;
        l = std::max(l, level[base(o)]);
      }
      level[x] = l;
    }
  }
  int nphase = 1;
  for (auto& kv : phase) nphase = std::max(nphase, kv.second + 1);
  for (auto& kv : level) nphase = std::max(nphase, kv.second + 1);
  if (nphase > RP_MAXPH) fail(E_INTERNAL, "row region has too many phases");
  // scalar registers
  std::map<int, int> sreg;
  int next_sreg = RP_SREG0;
  for (int x : order)
    if (rg.scalar.count(x) || rg.reduces.count(x)) {
      if (next_sreg >= RP_NREG) fail(E_INTERNAL, "row region needs too many per-row registers");
      sreg[x] = next_sreg++;
    }
  // external inputs (shared by all phases)
  std::map<int, int> in_index;
  int64_t bytes = 0;
  auto input_of = [&](int o) {
    auto it = in_index.find(o);
    if (it != in_index.end()) return it->second;
    if (P.nin >= RP_MAXIN) fail(E_INTERNAL, "row region has too many inputs");
    TView v = view_of(o);
    EwIn& in = P.in[P.nin];
    in.p = v.p;
    in.dt = v.dt;
    in.sel_dim = -1;
    for (int d = 0; d < P.rank; ++d) in.stride[d] = d < v.rank ? v.stride[d] : 0;
    bytes += g_.nodes[o].numel() * (int64_t)dt_size(g_.nodes[o].dt);
    in_index[o] = P.nin;
    return P.nin++;
  };
  int ncode = 0;
  auto emit = [&](const EwInstr& I) {
    if (ncode >= RP_MAXCODE) fail(E_INTERNAL, "row region program too long");
    P.code[ncode++] = I;
  };
  auto opcode = [&](const Node& n, EwInstr& I) {
    switch (n.op) {
      case Op::Add: I.op = EW_ADD; break;
      case Op::Sub: I.op = EW_SUB; break;
      case Op::Mul: I.op = EW_MUL; break;
      case Op::Div: I.op = EW_DIV; break;
      case Op::Max: I.op = EW_MAX; break;
      case Op::Min: I.op = EW_MIN; break;
      case Op::Exp: I.op = EW_EXP; break;
      case Op::Tanh: I.op = EW_TANH; break;
      case Op::Sqrt: I.op = EW_SQRT; break;
      case Op::Rsqrt: I.op = EW_RSQRT; break;
      case Op::Sin: I.op = EW_SIN; break;
      case Op::Cos: I.op = EW_COS; break;
      case Op::Logistic: I.op = EW_LOGISTIC; break;
      case Op::Neg: I.op = EW_NEG; break;
      case Op::Abs: I.op = EW_ABS; break;
      case Op::Convert: I.op = EW_CONVERT; I.aux = (uint8_t)kdt(g_.nodes[n.in[0]].dt); break;
      case Op::Compare: I.op = EW_CMP; I.aux = (uint8_t)n.i0; I.aux2 = (uint8_t)kdt(g_.nodes[n.in[0]].dt); break;
      case Op::Select: I.op = EW_SELECT; break;
      default: fail(E_INTERNAL, "not an elementwise op in a row region: " + n.name);
    }
  };
  std::vector<std::pair<int, int>> full_outs;  // (node, phase)
  // materialised members (needed outside the region or returned)
  // (directly, or through an alias view that is used outside or returned)
  std::function<bool(int)> materialised = [&](int x) {
    for (int o : g_.outputs)
      if (o == x) return true;
    for (int u : users_[x]) {
      if (!live_[u]) continue;
      if (region_of_[u] != rid) return true;
      if (rg.alias.count(u) && materialised(u)) return true;
    }
    return false;
  };
  for (int ph = 0; ph < nphase; ++ph) {
    RowPhase& Ph = P.ph[ph];
    Ph.red_reg = -1;
    Ph.lo = (uint16_t)ncode;
    // roots: reduce inputs of this phase, materialised full members of this phase
    std::vector<int> roots;
    int red = -1;
    for (int r : rg.reduces)
      if (phase[r] == ph) {
        if (red >= 0) fail(E_INTERNAL, "two reductions in one row phase");
        red = r;
        // a reduction of an external tensor reads it directly (loaded below)
        if (rg.full.count(g_.nodes[r].in[0])) roots.push_back(g_.nodes[r].in[0]);
      }
    for (int x : rg.full)
      if (phase[x] == ph && materialised(x)) roots.push_back(x);
    std::set<int> need;
    std::vector<int> st(roots.begin(), roots.end());
    while (!st.empty()) {
      int x = st.back();
      st.pop_back();
      if (need.count(x)) continue;
      need.insert(x);
      for (int o : g_.nodes[x].in) {
        int b = base(o);
        if (rg.full.count(b) && !is_splat(o)) st.push_back(b);
      }
    }
    // per-element program (registers 0..RP_SREG0-1 with reuse)
    std::map<int, int> reg;
    std::map<int, int> last_use;
    std::vector<int> list(need.begin(), need.end());
    std::sort(list.begin(), list.end());
    for (size_t k = 0; k < list.size(); ++k)
      for (int o : g_.nodes[list[k]].in) last_use[base(o)] = (int)k;
    std::set<int> pinned(roots.begin(), roots.end());
    std::vector<int> freeregs;
    for (int r = RP_SREG0 - 1; r >= 0; --r) freeregs.push_back(r);
    auto alloc = [&]() {
      if (freeregs.empty()) fail(E_INTERNAL, "row region needs too many registers");
      int r = freeregs.back();
      freeregs.pop_back();
      return r;
    };
    std::map<int, int> load_reg, imm_reg;
    for (size_t k = 0; k < list.size(); ++k) {
      int x = list[k];
      const Node& n = g_.nodes[x];
      std::vector<int> regs;
      for (int o : n.in) {
        if (is_splat(o)) {
          EwInstr I{};
          I.op = EW_IMM;
          I.dt = (uint8_t)kdt(g_.nodes[o].dt);
          I.dst = (uint8_t)alloc();
          I.fimm = (float)loc_[o].splat;
          I.iimm = (int32_t)(int64_t)loc_[o].splat;
          emit(I);
          regs.push_back(I.dst);
          continue;
        }
        int b = base(o);
        if (rg.full.count(b)) {
          regs.push_back(reg.at(b));
        } else if (sreg.count(b)) {
          regs.push_back(sreg.at(b));
        } else {
          auto it = load_reg.find(o);
          if (it == load_reg.end()) {
            EwInstr I{};
            I.op = EW_LOAD;
            int ii = input_of(o);
            I.dt = (uint8_t)P.in[ii].dt;
            I.aux = (uint8_t)ii;
            I.dst = (uint8_t)alloc();
            emit(I);
            it = load_reg.emplace(o, I.dst).first;
          }
          regs.push_back(it->second);
        }
      }
      EwInstr I{};
      opcode(n, I);
      I.dt = (uint8_t)kdt(n.dt);
      if (regs.size() > 0) I.a = (uint8_t)regs[0];
      if (regs.size() > 1) I.b = (uint8_t)regs[1];
      if (regs.size() > 2) I.c = (uint8_t)regs[2];
      I.dst = (uint8_t)alloc();
      emit(I);
      // immediates are single use; operand registers die at their last use
      for (size_t q = 0; q < n.in.size(); ++q) {
        int o = n.in[q];
        if (is_splat(o)) { freeregs.push_back(regs[q]); continue; }
        int b = base(o);
        if (rg.full.count(b) && last_use[b] == (int)k && !pinned.count(b)) freeregs.push_back(reg[b]);
      }
      reg[x] = I.dst;
    }
    if (red >= 0 && !rg.full.count(g_.nodes[red].in[0])) {
      int o = g_.nodes[red].in[0];
      auto it = load_reg.find(o);
      if (it == load_reg.end()) {
        EwInstr I{};
        I.op = EW_LOAD;
        int ii = input_of(o);
        I.dt = (uint8_t)P.in[ii].dt;
        I.aux = (uint8_t)ii;
        I.dst = (uint8_t)alloc();
        emit(I);
        it = load_reg.emplace(o, I.dst).first;
      }
      reg[o] = it->second;
    }
    Ph.hi = (uint16_t)ncode;
    if (red >= 0) {
      const Node& rn = g_.nodes[red];
      Ph.red_reg = (int8_t)reg.at(rn.in[0]);
      Ph.red_kind = (uint8_t)rn.i0;
      Ph.red_dst = (uint8_t)sreg.at(red);
      Ph.red_dt = (uint8_t)kdt(rn.dt);
      Ph.red_init = (float)loc_[rn.in[1]].splat;
    }
    for (int x : rg.full)
      if (phase[x] == ph && materialised(x)) {
        if (P.nout >= RP_MAXOUT) fail(E_INTERNAL, "row region has too many outputs");
        RowOut& o = P.out[P.nout++];
        o.p = slot_ptr(ensure_buf(x));
        o.dt = kdt(g_.nodes[x].dt);
        o.reg = (int16_t)reg.at(x);
        o.phase = (int8_t)ph;
        o.scalar = 0;
        bytes += g_.nodes[x].numel() * (int64_t)dt_size(g_.nodes[x].dt);
      }
    // per-row program of the scalars that become available after this phase
    Ph.slo = (uint16_t)ncode;
    for (int x : order) {
      if (!rg.scalar.count(x) || level[x] != ph + 1) continue;
      const Node& n = g_.nodes[x];
      std::vector<int> regs;
      int tmp = 0;
      for (int o : n.in) {
        if (is_splat(o)) {
          EwInstr I{};
          I.op = EW_IMM;
          I.dt = (uint8_t)kdt(g_.nodes[o].dt);
          I.dst = (uint8_t)(tmp++);  // per-element registers are free between phases
          I.fimm = (float)loc_[o].splat;
          I.iimm = (int32_t)(int64_t)loc_[o].splat;
          emit(I);
          regs.push_back(I.dst);
        } else {
          regs.push_back(sreg.at(base(o)));
        }
      }
      EwInstr I{};
      opcode(n, I);
      I.dt = (uint8_t)kdt(n.dt);
      if (regs.size() > 0) I.a = (uint8_t)regs[0];
      if (regs.size() > 1) I.b = (uint8_t)regs[1];
      if (regs.size() > 2) I.c = (uint8_t)regs[2];
      I.dst = (uint8_t)sreg.at(x);
      emit(I);
    }
    Ph.shi = (uint16_t)ncode;
  }
  P.nphase = nphase;
  for (int x : order)
    if ((rg.scalar.count(x) || rg.reduces.count(x)) && materialised(x)) {
      if (P.nout >= RP_MAXOUT) fail(E_INTERNAL, "row region has too many outputs");
      RowOut& o = P.out[P.nout++];
      o.p = slot_ptr(ensure_buf(x));
      o.dt = kdt(g_.nodes[x].dt);
      o.reg = (int16_t)sreg.at(x);
      o.scalar = 1;
      bytes += P.rows * (int64_t)dt_size(g_.nodes[x].dt);
    }
  std::string label = "row:" + g_.nodes[rg.root].name;
  push(K_ROWNORM, blob_of(P), label, bytes);
}

// The printed argmax over the last axis of x (tensor.clj:519-532):
//   reduce_max_i32( convert_i32( compare_EQ(x, broadcast(reduce_max(x))) ) * broadcast(iota literal) )
// Returns x when node r is the final reduce of that chain, else -1.
int Planner::match_argmax(int r) const {
  const Node& R = g_.nodes[r];
  if (R.op != Op::Reduce || R.i0 != RED_MAX || R.dt != DT::I32 || R.in.size() != 2) return -1;
  const Node& M = g_.nodes[R.in[0]];
  const int rank = M.rank();
  if (M.op != Op::Mul || M.dt != DT::I32 || rank < 1 || R.ia.size() != 1 || R.ia[0] != rank - 1) return -1;
  double init;
  if (!const_cast<Planner*>(this)->splat_value(R.in[1], init) || init > 0) return -1;
  const int64_t V = M.shape.back();
  auto strip = [&](int n) {  // through reshapes and broadcasts
    while (g_.nodes[n].op == Op::Reshape || g_.nodes[n].op == Op::Broadcast) n = g_.nodes[n].in[0];
    return n;
  };
  // a chain of reshapes / broadcasts that only adds or repeats leading dims,
  // keeping the last axis: the value at (..., j) is the source's element j
  auto keeps_last = [&](int n, int src) {
    for (; n != src; n = g_.nodes[n].in[0]) {
      const Node& a = g_.nodes[n];
      const Node& b = g_.nodes[a.in[0]];
      if (b.shape.empty() || b.shape.back() != V) return false;
      for (size_t d = 0; d + 1 < b.shape.size(); ++d)
        if (b.shape[d] != 1) return false;
      if (a.op == Op::Broadcast && (a.ia.empty() || a.ia.back() != a.rank() - 1)) return false;
    }
    return true;
  };
  for (int side = 0; side < 2; ++side) {
    const Node& C = g_.nodes[M.in[side]];
    const int io = M.in[1 - side];
    if (C.op != Op::Convert || g_.nodes[C.in[0]].op != Op::Compare) continue;
    const Node& E = g_.nodes[C.in[0]];
    if (E.i0 != CMP_EQ) continue;
    // the index operand: an i32 literal 0 .. V-1 along the last axis
    const int ic = strip(io);
    const Node& K = g_.nodes[ic];
    if (K.op != Op::Constant || K.dt != DT::I32 || K.splat || K.numel() != V || !keeps_last(io, ic)) continue;
    const int32_t* kv = (const int32_t*)K.data.data();
    if (K.data.size() != (size_t)V * 4) continue;
    bool iota = true;
    for (int64_t j = 0; j < V && iota; ++j) iota = kv[j] == j;
    if (!iota) continue;
    // x compared with the broadcast of its own row maximum
    for (int e = 0; e < 2; ++e) {
      const int x = E.in[e], bm = E.in[1 - e];
      const Node& X = g_.nodes[x];
      if (!dt_is_float(X.dt) || X.shape != M.shape) continue;
      const int mx = strip(bm);
      const Node& Mx = g_.nodes[mx];
      if (Mx.op != Op::Reduce || Mx.i0 != RED_MAX || Mx.in[0] != x || Mx.ia.size() != 1 || Mx.ia[0] != rank - 1)
        continue;
      double minit;
      if (!const_cast<Planner*>(this)->splat_value(Mx.in[1], minit) || minit > -1e30) continue;
      // the row maximum at every position of its row: broadcast(reshape(mx) to
      // [..., 1]) with identity dimensions, or broadcast(mx) over the last axis
      std::vector<int64_t> lead(M.shape.begin(), M.shape.end() - 1), lead1 = lead;
      lead1.push_back(1);
      const Node& B = g_.nodes[bm];
      if (B.op != Op::Broadcast || Mx.shape != lead) continue;
      const Node& Bi = g_.nodes[B.in[0]];
      bool ok = false;
      if (B.in[0] == mx) {
        ok = (int)B.ia.size() == rank - 1;
        for (int d = 0; d < rank - 1 && ok; ++d) ok = B.ia[d] == d;
      } else if (Bi.op == Op::Reshape && Bi.in[0] == mx && Bi.shape == lead1) {
        ok = (int)B.ia.size() == rank;
        for (int d = 0; d < rank && ok; ++d) ok = B.ia[d] == d;
      }
      if (!ok) continue;
      // logits widened to f32 only for the comparison: the kernel reads the
      // narrower values (the widening is exact, so the result is the same)
      if (X.op == Op::Convert && (g_.nodes[X.in[0]].dt == DT::BF16 || g_.nodes[X.in[0]].dt == DT::F16) &&
          X.dt == DT::F32 && g_.nodes[X.in[0]].shape == X.shape)
        return X.in[0];
      return x;
    }
  }
  return -1;
}

void Planner::emit_attention(int d2) {
  const AttnMatch& am = attn_.at(d2);
  const Node& D2 = g_.nodes[d2];
  const Node& K = g_.nodes[am.kc];
  int oslot = ensure_buf(d2);
  AttnParams P{};
  P.q = view_of(am.q);
  P.k = view_of(am.kc);
  P.v = view_of(am.vc);
  if (mask_form_.count(d2)) {
    const MaskForm& f = mask_form_.at(d2);
    P.mask_mode = 1;
    P.mask_gt = (int32_t)f.gt;
    P.mask_lt = f.has_lt ? (int32_t)f.lt : INT32_MIN;
    P.mask_off = (int32_t)f.off;
    P.mask_mv = f.mv;
    P.mask_z = f.z;
    if (f.pos_param >= 0) {
      P.mask_pos = view_of(f.pos_param).p;
      P.has_mask_pos = 1;
    }
    // a view whose row offset is the query index (never dereferenced)
    P.mask = P.q;
    P.mask.dt = kdt(DT::F32);
    P.mask.rank = 4;
    const int64_t shp[4] = {D2.shape[0], D2.shape[1], D2.shape[2], K.shape[2]}, str[4] = {0, 0, 1, 0};
    for (int i = 0; i < 4; ++i) {
      P.mask.shape[i] = shp[i];
      P.mask.stride[i] = str[i];
    }
    plan_.n_mask_computed++;
    if (getenv("CLJXLA_B200_DEBUG_ATTN"))
      fprintf(stderr, "attention %s: computed mask gt %lld lt %s%lld off %lld mv %g z %g pos %s\n", D2.name.c_str(),
              (long long)f.gt, f.has_lt ? "" : "none ", (long long)f.lt, (long long)f.off, (double)f.mv, (double)f.z,
              f.pos_param >= 0 ? g_.nodes[f.pos_param].name.c_str() : "-");
  } else {
    P.mask = view_of(am.mask);
  }
  P.B = (int32_t)D2.shape[0];
  P.nq = (int32_t)D2.shape[1];
  P.Sq = (int32_t)D2.shape[2];
  P.hd = (int32_t)D2.shape[3];
  P.nkv = (int32_t)K.shape[1];
  P.T = (int32_t)K.shape[2];
  P.group = am.group;
  const int hpl = P.hd / 32;
  // K/V rows must be contiguous along hd and aligned for hd/32-element vector loads
  auto kv_ok = [&](const TView& v) {
    int64_t es = (int64_t)dt_size((DT)v.dt);
    bool ok = v.stride[3] == 1 && (v.p.off % (hpl * es)) == 0;
    for (int d = 0; d < 3; ++d) ok &= (v.stride[d] % hpl) == 0;
    return ok;
  };
  if (!kv_ok(P.k)) P.k = materialize(P.k, K.shape, K.dt);
  if (!kv_ok(P.v)) P.v = materialize(P.v, g_.nodes[am.vc].shape, g_.nodes[am.vc].dt);
  P.k_dt = P.k.dt;
  P.dt_d1 = kdt(g_.nodes[am.d1].dt);
  P.dt_m = kdt(g_.nodes[am.m].dt);
  P.dt_sub = kdt(g_.nodes[am.sub].dt);
  P.dt_exp = kdt(g_.nodes[am.exp].dt);
  P.out_dt = kdt(D2.dt);
  P.mask_skip = -5000.0f;
  // the score chain as a register program; register 0 holds the incoming score
  int nreg = 1, cur = 0;
  auto emit = [&](const EwInstr& I) {
    if (P.nchain >= 12) fail(E_INTERNAL, "attention score chain too long");
    P.chain[P.nchain++] = I;
  };
  for (int c : am.chain) {
    const Node& C = g_.nodes[c];
    std::vector<int> regs;
    for (int o : C.in) {
      double v;
      if (splat_value(o, v)) {
        EwInstr I{};
        I.op = EW_IMM;
        I.dt = (uint8_t)kdt(DT::F32);
        I.dst = (uint8_t)nreg++;
        I.fimm = (float)v;
        emit(I);
        regs.push_back(I.dst);
      } else {
        regs.push_back(cur);
      }
    }
    EwInstr I{};
    switch (C.op) {
      case Op::Mul: I.op = EW_MUL; break;
      case Op::Div: I.op = EW_DIV; break;
      case Op::Add: I.op = EW_ADD; break;
      case Op::Sub: I.op = EW_SUB; break;
      case Op::Max: I.op = EW_MAX; break;
      case Op::Min: I.op = EW_MIN; break;
      case Op::Tanh: I.op = EW_TANH; break;
      case Op::Neg: I.op = EW_NEG; break;
      default: I.op = EW_CONVERT; break;
    }
    I.dt = (uint8_t)kdt(C.dt);
    I.a = (uint8_t)regs[0];
    I.b = (uint8_t)(regs.size() > 1 ? regs[1] : 0);
    I.dst = (uint8_t)nreg++;
    if (nreg > 16) fail(E_INTERNAL, "attention score chain needs too many registers");
    emit(I);
    cur = I.dst;
  }
  P.chain_out = cur;
  if (getenv("CLJXLA_B200_DEBUG_ATTN")) {
    fprintf(stderr, "attention chain (%d ops, out r%d):", P.nchain, P.chain_out);
    for (int i = 0; i < P.nchain; ++i)
      fprintf(stderr, " [op %d dt %d r%d <- r%d r%d imm %g]", P.chain[i].op, P.chain[i].dt, P.chain[i].dst,
              P.chain[i].a, P.chain[i].b, P.chain[i].fimm);
    fprintf(stderr, " dt_d1 %d dt_m %d dt_sub %d dt_exp %d\n", P.dt_d1, P.dt_m, P.dt_sub, P.dt_exp);
  }
  {
    // closed forms: trailing converts to f32 change no float value (the kernels
    // hold f32), so drop them; then nothing (identity) or one multiply by a constant
    int n = P.nchain, out = P.chain_out;
    while (n > 0 && P.chain[n - 1].op == EW_CONVERT && P.chain[n - 1].dt == KDT_F32 && P.chain[n - 1].dst == out) {
      out = P.chain[n - 1].a;
      --n;
    }
    if (n == 0 && out == 0) {
      P.chain_kind = 2;
    } else if (n == 2 && P.chain[0].op == EW_IMM && P.chain[1].op == EW_MUL && out == P.chain[1].dst &&
               ((P.chain[1].a == 0 && P.chain[1].b == P.chain[0].dst) ||
                (P.chain[1].b == 0 && P.chain[1].a == P.chain[0].dst))) {
      P.chain_kind = 1;
      P.chain_c = P.chain[0].fimm;
      P.chain_dt = P.chain[1].dt;
    }
  }
  const int64_t rows_kv = (int64_t)P.B * P.nkv;
  P.qtile = P.Sq == 1 ? 1 : std::max(1, std::min(P.Sq, 8 / P.group));
  if (P.qtile * P.group > 8) P.qtile = 1;
  if (P.group > 8) fail(E_UNIMPLEMENTED, "attention with more than 8 query heads per KV head");
  int64_t qtiles = (P.Sq + P.qtile - 1) / P.qtile;
  int64_t ctas = rows_kv * qtiles;
  // one 128-position round per warp-group of a CTA, at most two CTAs per SM;
  // the tensor-core decode kernel takes 64-position splits
  P.use_tc = attention_tc_ok(P) && !getenv_off("CLJXLA_B200_ATTN_TC") ? 1 : 0;
  if (!P.use_tc && P.Sq > P.qtile && attention_tc_prefill_ok(P) && !getenv_off("CLJXLA_B200_ATTN_TC")) P.use_tc = 2;
  int64_t per_split = P.use_tc ? 64 : 128;
  if (const char* e = getenv("CLJXLA_B200_ATTN_SPLIT"))  // positions per split (measurement sweeps)
    if (atoi(e) >= 16) per_split = atoi(e);
  int splits = (int)std::min<int64_t>((P.T + per_split - 1) / per_split, std::max<int64_t>(1, 2 * 148 / ctas));
  splits = std::max(1, std::min(splits, ATTN_MERGE_MAX_SPLITS));
  if (P.use_tc == 2) splits = 1;  // whole rows per CTA
  if (getenv("CLJXLA_B200_DEBUG_ATTN"))
    fprintf(stderr, "attention %s: Sq %d T %d use_tc %d chain_kind %d chain_dt %d mask dt %d off %lld strides %lld %lld %lld %lld\n",
            D2.name.c_str(), P.Sq, P.T, P.use_tc, P.chain_kind, P.chain_dt, P.mask.dt, (long long)P.mask.p.off,
            (long long)P.mask.stride[0], (long long)P.mask.stride[1], (long long)P.mask.stride[2],
            (long long)P.mask.stride[3]);
  P.splits = splits;
  if (P.Sq == 1 && attention_dec_ok(P) && !getenv_off("CLJXLA_B200_ATTN_DEC")) {
    P.use_tc = 3;
    plan_attention_dec(P, 148);
    P.dec_live_splits = P.mask_mode && P.mask_mv <= P.mask_skip && P.mask_z > P.mask_skip &&
                        !getenv_off("CLJXLA_B200_ATTN_LIVE_SPLITS");
    splits = P.splits;
    if (getenv("CLJXLA_B200_DEBUG_ATTN"))
      fprintf(stderr, "attention %s: staged decode, %d splits of %d positions, chunk %d\n", D2.name.c_str(), P.splits,
              P.dec_per_split, P.dec_chunk);
  }
  P.out = slot_ptr(oslot);
  int64_t kvbytes = 2 * (int64_t)P.B * P.nkv * P.T * P.hd * (int64_t)dt_size((DT)P.k_dt);
  int64_t rows = (int64_t)P.B * P.nq * P.Sq;
  if (splits > 1) {
    P.part = slot_ptr(new_tmp(attention_part_bytes(P)));
    // arrival counters (zero in the uploaded constant blob, reset by the merging CTA)
    const int64_t groups = rows_kv * qtiles;
    size_t off = (plan_.const_blob.size() + 255) & ~size_t(255);
    plan_.const_blob.resize(off + 4 * groups, 0);
    P.counters = slot_ptr(P_ + O_ + U_, (int64_t)off);
    P.use_counters = 1;
  }
  push(K_ATTN_DECODE, blob_of(P), D2.name, kvbytes, 4LL * rows * P.T * P.hd);
}

bool Planner::splat_value(int n, double& v) {
  // evaluated on the graph: the chain's constants are dead once the block is fused
  const Node& nd = g_.nodes[n];
  if (nd.op == Op::Constant) {
    if (!nd.splat) return false;
    v = nd.splat_val;
    return true;
  }
  if (is_view_op(nd, g_)) return splat_value(nd.in[0], v);
  if (nd.op == Op::Convert && dt_is_float(nd.dt) && splat_value(nd.in[0], v)) {
    v = round_host(v, nd.dt);
    return true;
  }
  return false;
}

void Planner::emit_node_kernel(int id) {
  const Node& n = g_.nodes[id];
  if (attn_.count(id)) {
    emit_attention(id);
    return;
  }
  int oslot = ensure_buf(id);
  switch (n.op) {
    case Op::Reduce: {
      if (argmax_.count(id)) {
        const int x = argmax_.at(id);
        ArgmaxParams A{};
        A.in = view_of(x);
        A.out = slot_ptr(oslot);
        A.V = g_.nodes[x].shape.back();
        A.rows = g_.nodes[x].numel() / std::max<int64_t>(1, A.V);
        // a wave of CTAs over all rows, at least 2048 logits per CTA
        A.ctas = (int32_t)std::max<int64_t>(1, std::min<int64_t>((2 * 148 + A.rows - 1) / A.rows, A.V / 2048));
        A.ctas = std::min<int32_t>(A.ctas, 1024);
        if (A.ctas > 1) {
          A.part = slot_ptr(new_tmp(argmax_part_bytes(A)));
          size_t off = (plan_.const_blob.size() + 255) & ~size_t(255);
          plan_.const_blob.resize(off + 4 * A.rows, 0);
          A.counters = slot_ptr(P_ + O_ + U_, (int64_t)off);
        }
        push(K_ARGMAX, blob_of(A), n.name, g_.nodes[x].numel() * (int64_t)dt_size(g_.nodes[x].dt) + A.rows * 4);
        break;
      }
      const Node& in = g_.nodes[n.in[0]];
      if (!is_splat(n.in[1])) fail(E_UNIMPLEMENTED, "reduce with a non-constant init value");
      TView v = view_of(n.in[0]);
      ReduceParams R{};
      R.in = v;
      R.out = slot_ptr(oslot);
      R.out_dt = kdt(n.dt);
      R.kind = (int)n.i0;
      R.init = (float)loc_[n.in[1]].splat;
      std::set<int> red(n.ia.begin(), n.ia.end());
      R.n_out = 1;
      R.n_red = 1;
      for (int d = 0; d < in.rank(); ++d) {
        if (red.count(d)) {
          R.red_shape[R.nred] = in.shape[d];
          R.red_stride[R.nred] = v.stride[d];
          R.nred++;
          R.n_red *= in.shape[d];
        } else {
          R.keep_shape[R.nkeep] = in.shape[d];
          R.keep_stride[R.nkeep] = v.stride[d];
          R.nkeep++;
          R.n_out *= in.shape[d];
        }
      }
      if (R.nred == 0) { R.red_shape[0] = 1; R.red_stride[0] = 0; R.nred = 1; }
      push(K_REDUCE, blob_of(R), n.name,
           in.numel() * (int64_t)dt_size(in.dt) + n.numel() * (int64_t)dt_size(n.dt));
      break;
    }
    case Op::Gather: {
      const Node& tab = g_.nodes[n.in[0]];
      const Node& idx = g_.nodes[n.in[1]];
      bool ok = tab.rank() == 2 && n.ib == std::vector<int64_t>{0} && n.ic == std::vector<int64_t>{0} &&
                n.id.size() == 2 && n.id[0] == 1 && n.id[1] == tab.shape[1] && idx.rank() >= 1 &&
                n.i0 == idx.rank() - 1 && idx.shape.back() == 1 && n.ia == std::vector<int64_t>{idx.rank() - 1} &&
                (tab.dt == DT::F32 || tab.dt == DT::BF16 || tab.dt == DT::F16);
      if (!ok) fail(E_UNIMPLEMENTED, "gather form not supported (only row gathers of a 2-D table)");
      TView tv = view_of(n.in[0]);
      if (tv.stride[1] != 1) tv = materialize(tv, tab.shape, tab.dt);
      GatherParams G{};
      G.table = tv.p;
      G.table_dt = tv.dt;
      G.rows_table = tab.shape[0];
      G.row_len = tab.shape[1];
      G.table_row_stride = tv.stride[0];
      TView iv = view_of(n.in[1]);
      G.idx = iv;
      G.idx_dt = iv.dt;
      G.out = slot_ptr(oslot);
      G.n_rows = idx.numel();
      push(K_GATHER, blob_of(G), n.name, 2 * n.numel() * (int64_t)dt_size(n.dt));
      break;
    }
    case Op::DUS: {
      DusParams D{};
      D.rank = n.rank();
      D.dt = kdt(n.dt);
      D.operand = view_of(n.in[0]);
      D.update = view_of(ins_[id][1]);  // may be the unconverted value (rounded on store)
      const Node& up = g_.nodes[ins_[id][1]];
      for (int d = 0; d < D.rank; ++d) {
        D.out_shape[d] = n.shape[d];
        D.upd_shape[d] = up.shape[d];
        int s = n.in[2 + d];
        if (is_splat(s)) {
          D.start_imm[d] = (int64_t)loc_[s].splat;
        } else {
          TView sv = view_of(s);
          D.start_ptr[d] = sv.p;
          D.start_dt[d] = sv.dt;
          D.start_is_ptr[d] = 1;
        }
      }
      D.out = slot_ptr(oslot);
      D.n = n.numel();
      int64_t ub = up.numel() * (int64_t)dt_size(n.dt);
      auto ip = inplace_of_.find(id);
      if (ip != inplace_of_.end()) {
        // in place over the argument's storage (the result slot points at it)
        const InplaceDus& d = plan_.inplace[ip->second];
        D.operand = dense_view(oslot, n.dt, n.shape);
        D.in_place = 1;
        D.has_undo = 1;
        D.undo = slot_ptr(d.undo_slot);
        push(K_DUS, blob_of(D), n.name, 2 * ub);
        break;
      }
      if (D.operand.dt == D.dt) {
        // copy the operand with the vectorised copy, then write the window in place
        CopyParams C{};
        C.src = D.operand;
        C.dst = dense_view(oslot, n.dt, n.shape);
        C.n = n.numel();
        push(K_COPY, blob_of(C), n.name + ".copy", 2 * n.numel() * (int64_t)dt_size(n.dt));
        D.operand = C.dst;
        D.in_place = 1;
        push(K_DUS, blob_of(D), n.name, ub);
        break;
      }
      push(K_DUS, blob_of(D), n.name, 2 * n.numel() * (int64_t)dt_size(n.dt) + ub);
      break;
    }
    case Op::Concat: {
      int64_t off = 0;
      int dim = (int)n.i0;
      TView ov = dense_view(oslot, n.dt, n.shape);
      for (int x : n.in) {
        const Node& xn = g_.nodes[x];
        CopyParams C{};
        C.dst = ov;
        for (int d = 0; d < C.dst.rank; ++d) C.dst.shape[d] = xn.shape[d];
        C.dst.p.off += off * ov.stride[dim] * (int64_t)dt_size(n.dt);
        if (is_splat(x)) {
          // broadcast a splat into the slice through a one-instruction program
          EwParams E{};
          E.rank = xn.rank();
          E.n = xn.numel();
          for (int d = 0; d < E.rank; ++d) E.dims[d] = xn.shape[d];
          EwInstr I{};
          I.op = EW_IMM;
          I.dt = (uint8_t)kdt(xn.dt);
          I.fimm = (float)loc_[x].splat;
          I.iimm = (int32_t)(int64_t)loc_[x].splat;
          E.code[0] = I;
          E.ncode = 1;
          // write through a strided copy afterwards is overkill; store densely into a scratch then copy
          int slot = new_tmp(xn.numel() * (int64_t)dt_size(xn.dt));
          E.out[0].p = slot_ptr(slot);
          E.out[0].dt = kdt(xn.dt);
          E.out[0].reg = 0;
          E.nout = 1;
          push(K_EW, blob_of(E), n.name + ".splat");
          C.src = dense_view(slot, xn.dt, xn.shape);
        } else {
          C.src = view_of(x);
        }
        C.n = xn.numel();
        push(K_COPY, blob_of(C), n.name, 2 * C.n * (int64_t)dt_size(n.dt));
        off += xn.shape[dim];
      }
      break;
    }
    case Op::AllReduce: {
      // NCCL reads and writes plain device addresses: a dense arena copy of the
      // operand in, the arena result slot out (both fixed for the executable)
      const Node& in = g_.nodes[n.in[0]];
      const int red = n.ia.empty() ? RED_ADD : (int)n.ia[0];
      if (!(n.dt == DT::F32 || n.dt == DT::BF16 || n.dt == DT::F16 || (red == RED_MAX && n.dt == DT::I32)) ||
          in.dt != n.dt)
        fail(E_UNIMPLEMENTED, "all_reduce of element type " + std::string(dt_name(n.dt)));
      TView v = view_of(n.in[0]);
      bool dense = v.p.slot >= tmp_slot(0) && v.p.off % 16 == 0;
      int64_t acc = 1;
      for (int d = v.rank - 1; d >= 0 && dense; --d) {
        if (v.shape[d] != 1 && v.stride[d] != acc) dense = false;
        acc *= v.shape[d];
      }
      if (!dense) v = materialize(v, in.shape, in.dt);
      AllReduceParams A{};
      A.src = v.p;
      A.dst = slot_ptr(oslot);
      A.count = n.numel();
      A.dt = kdt(n.dt);
      A.ranks = (int32_t)n.i0;
      A.reduce = red;
      push(K_ALLREDUCE, blob_of(A), n.name, 2 * n.numel() * (int64_t)dt_size(n.dt));
      break;
    }
    case Op::Dot: {
      int64_t bytes = 0, flops = 0;
      if (opt_.fast_kernels && !getenv_off("CLJXLA_B200_SPLIT_GEMM") && emit_split_dot(id, oslot)) break;
      GemmParams G = dot_params(id, oslot, &bytes, &flops);
      Launch fl;
      TcGemmParams tc;
      if (opt_.fast_kernels && make_gemv(G, fl)) {
        fl.label = n.name;
        fl.algo_bytes = bytes;
        fl.algo_flops = flops;
        // the other projections of the same input (q / k / v, gate / up) join this launch
        for (int u : users_[n.in[0]]) {
          if (u == id || !live_[u] || g_.nodes[u].op != Op::Dot || pre_emitted_.count(u) || attn_.count(u) ||
              loc_[u].kind != Loc::BUF)
            continue;
          const Node& un = g_.nodes[u];
          if (un.in[0] != n.in[0] || un.ia != n.ia || un.ic != n.ic) continue;
          const Node& wn = g_.nodes[view_root(un.in[1])];
          if (wn.op != Op::Param && wn.op != Op::Constant) continue;
          if (emitted_units_.count(u)) continue;
          int64_t ub = 0, uf = 0;
          GemmParams GU = dot_params(u, ensure_buf(u), &ub, &uf);
          if (!gemv_add_segment(fl, GU)) continue;
          pre_emitted_.insert(u);
          fl.label += "," + un.name;
          fl.algo_bytes += ub;
          fl.algo_flops += uf;
        }
        plan_.launches.push_back(std::move(fl));
      } else if (opt_.fast_kernels && !getenv_off("CLJXLA_B200_TC_GEMM") && make_tc_gemm(G, tc)) {
        int bm, bn, bk;
        tc_gemm_tile_shape(&bm, &bn, &bk);
        TmapSpec ta, tb;
        ta.base = G.a;
        ta.inner = G.K;
        ta.outer = G.M;
        ta.row_bytes = G.a_sm * 2;
        ta.box_inner = bk;
        ta.box_outer = bm;
        tb.base = G.b;
        tb.inner = G.K;
        tb.outer = G.N;
        tb.row_bytes = G.b_sn * 2;
        tb.box_inner = bk;
        tb.box_outer = bn;
        tc_tiling(tc, ta, tb);
        tc.tmap_a_index = (int32_t)plan_.tmaps.size();
        plan_.tmaps.push_back(ta);
        tc.tmap_b_index = (int32_t)plan_.tmaps.size();
        plan_.tmaps.push_back(tb);
        push(K_GEMM_TC, blob_of(tc), n.name, bytes, flops);
      } else {
        push(K_GEMM, blob_of(G), n.name, bytes, flops);
      }
      break;
    }
    default:
      fail(E_UNIMPLEMENTED, std::string("no kernel for op ") + op_name(n.op));
  }
}

// f32 activations [M, K] times a bf16 weight [N, K] with M >= 16 (a prefill
// attention-output projection): one elementwise program reads the activation
// through its printed view and writes it as three exact bf16 planes
// hi / mid / lo; the tensor-core GEMM then accumulates the three plane
// products in f32.  Nothing is emitted unless both launches apply.
bool Planner::emit_split_dot(int id, int oslot) {
  const Node& n = g_.nodes[id];
  const Node& a = g_.nodes[n.in[0]];
  const Node& b = g_.nodes[n.in[1]];
  if (a.dt != DT::F32 || b.dt != DT::BF16 || !(n.dt == DT::F32 || n.dt == DT::BF16)) return false;
  auto has = [](const std::vector<int64_t>& v, int64_t d) { return std::find(v.begin(), v.end(), d) != v.end(); };
  for (int64_t d : n.ia)
    if (a.shape[d] != 1) return false;
  for (int64_t d : n.ib)
    if (b.shape[d] != 1) return false;
  std::vector<int64_t> lf, rf;
  int64_t M = 1, K = 1, N = 1;
  for (int d = 0; d < a.rank(); ++d)
    if (!has(n.ia, d) && !has(n.ic, d)) lf.push_back(d), M *= a.shape[d];
  for (int64_t d : n.ic) K *= a.shape[d];
  for (int d = 0; d < b.rank(); ++d)
    if (!has(n.ib, d) && !has(n.id, d)) rf.push_back(d), N *= b.shape[d];
  if (M < 16 || N < 16 || K < 16 || (K % 8) || (int)(lf.size() + n.ic.size()) > CLJXLA_MAXR) return false;
  // the weight: contracting dims collapse to unit stride, free dims to one row stride
  TView bv = view_of(n.in[1]);
  auto collapse = [&](const std::vector<int64_t>& dims, int64_t& stride) {
    int64_t prev = -1;
    stride = 0;
    for (int64_t d : dims) {
      if (bv.shape[d] == 1) continue;
      if (prev >= 0 && prev != bv.stride[d] * bv.shape[d]) return false;
      prev = bv.stride[d];
    }
    stride = prev < 0 ? 0 : prev;
    return true;
  };
  int64_t sk = 0, sn = 0;
  if (!collapse(n.id, sk) || !collapse(rf, sn) || sk != 1) return false;
  GemmParams G{};
  G.batch = 1;
  G.M = M;
  G.N = N;
  G.K = K;
  G.a_dt = KDT_F32;
  G.b_dt = KDT_BF16;
  G.c_dt = kdt(n.dt);
  G.b = bv.p;
  G.b_sk = 1;
  G.b_sn = sn;
  G.c = slot_ptr(oslot);
  TcGemmParams tc;
  if (!make_tc_gemm_split(G, tc)) return false;
  // the three planes: rows in the printed free-dim order, K in contracting order
  EwParams E{};
  E.rank = 0;
  bool natural = true;  // [M, K] row-major is the operand's own element order
  {
    int k = 0;
    for (int d = 0; d < a.rank(); ++d) {
      if (has(n.ia, d)) continue;
      const int64_t want = k < (int)lf.size() ? lf[k] : n.ic[k - lf.size()];
      if (want != d) natural = false;
      ++k;
    }
  }
  int src = n.in[0];
  // a reshape of a permuted view (the heads of an attention context merged
  // into K) keeps the element order: read the reshape's operand directly
  // instead of materialising it
  while (natural && g_.nodes[src].op == Op::Reshape && loc_[src].kind == Loc::VIEWOP && mat_slot_[src] < 0 &&
         g_.nodes[g_.nodes[src].in[0]].rank() <= CLJXLA_MAXR)
    src = g_.nodes[src].in[0];
  TView av = view_of(src);
  if (src != n.in[0]) {
    for (int d = 0; d < av.rank; ++d) E.dims[E.rank] = av.shape[d], E.in[0].stride[E.rank++] = av.stride[d];
  } else {
    for (int64_t d : lf) E.dims[E.rank] = a.shape[d], E.in[0].stride[E.rank++] = av.stride[d];
    for (int64_t d : n.ic) E.dims[E.rank] = a.shape[d], E.in[0].stride[E.rank++] = av.stride[d];
  }
  E.n = M * K;
  E.in[0].p = av.p;
  E.in[0].dt = av.dt;
  E.in[0].sel_dim = -1;
  E.nin = 1;
  auto op = [&](int opc, int dt, int dst, int x, int y, int aux) {
    EwInstr I{};
    I.op = (uint8_t)opc;
    I.dt = (uint8_t)dt;
    I.dst = (uint8_t)dst;
    I.a = (uint8_t)x;
    I.b = (uint8_t)y;
    I.aux = (uint8_t)aux;
    E.code[E.ncode++] = I;
  };
  op(EW_LOAD, KDT_F32, 0, 0, 0, 0);
  op(EW_CONVERT, KDT_BF16, 1, 0, 0, KDT_F32);  // hi
  op(EW_SUB, KDT_F32, 2, 0, 1, 0);             // exact remainder
  op(EW_CONVERT, KDT_BF16, 3, 2, 0, KDT_F32);  // mid
  op(EW_SUB, KDT_F32, 4, 2, 3, 0);
  op(EW_CONVERT, KDT_BF16, 5, 4, 0, KDT_F32);  // lo
  const int64_t plane = M * K * 2;
  const int slot = new_tmp(3 * plane);
  for (int p = 0; p < 3; ++p) {
    E.out[p].p = slot_ptr(slot, p * plane);
    E.out[p].dt = KDT_BF16;
    E.out[p].reg = 1 + 2 * p;
  }
  E.nout = 3;
  push(K_EW, blob_of(E), n.name + ".planes", M * K * 4 + 3 * plane);
  tc.a = slot_ptr(slot);
  int bm, bn, bk;
  tc_gemm_tile_shape(&bm, &bn, &bk);
  TmapSpec ta, tb;
  ta.base = tc.a;
  ta.inner = K;
  ta.outer = 3 * M;
  ta.row_bytes = K * 2;
  ta.box_inner = bk;
  ta.box_outer = bm;
  tb.base = G.b;
  tb.inner = K;
  tb.outer = N;
  tb.row_bytes = sn * 2;
  tb.box_inner = bk;
  tb.box_outer = bn;
  tc_tiling(tc, ta, tb);
  tc.tmap_a_index = (int32_t)plan_.tmaps.size();
  plan_.tmaps.push_back(ta);
  tc.tmap_b_index = (int32_t)plan_.tmaps.size();
  plan_.tmaps.push_back(tb);
  push(K_GEMM_TC, blob_of(tc), n.name,
       a.numel() * 4 + b.numel() * 2 + n.numel() * (int64_t)dt_size(n.dt), 2 * M * N * K);
  return true;
}

GemmParams Planner::dot_params(int id, int oslot, int64_t* bytes_out, int64_t* flops_out) {
  const Node& n = g_.nodes[id];
  {
    {
      const Node& a = g_.nodes[n.in[0]];
      const Node& b = g_.nodes[n.in[1]];
      std::vector<int64_t> lb = n.ia, rb = n.ib, lc = n.ic, rc = n.id, lf, rf;
      for (int d = 0; d < a.rank(); ++d)
        if (std::find(lb.begin(), lb.end(), d) == lb.end() && std::find(lc.begin(), lc.end(), d) == lc.end())
          lf.push_back(d);
      for (int d = 0; d < b.rank(); ++d)
        if (std::find(rb.begin(), rb.end(), d) == rb.end() && std::find(rc.begin(), rc.end(), d) == rc.end())
          rf.push_back(d);
      auto collapse = [](const TView& v, const std::vector<int64_t>& dims, int64_t& size, int64_t& stride) {
        size = 1;
        stride = 0;
        int64_t prev_stride = -1, prev_size = 1;
        bool first = true;
        for (int64_t d : dims) {
          int64_t s = v.shape[d];
          size *= s;
          if (s == 1) continue;
          if (!first && prev_stride != v.stride[d] * s) return false;
          prev_stride = v.stride[d];
          prev_size = s;
          first = false;
        }
        (void)prev_size;
        stride = first ? 0 : prev_stride;
        return true;
      };
      auto canon = [&](int x, const std::vector<int64_t>& g1, const std::vector<int64_t>& g2,
                       const std::vector<int64_t>& g3, int64_t s[3], int64_t z[3]) {
        TView v = view_of(x);
        const Node& xn = g_.nodes[x];
        bool ok = collapse(v, g1, z[0], s[0]) && collapse(v, g2, z[1], s[1]) && collapse(v, g3, z[2], s[2]);
        if (!ok) {
          // permuted dense copy in (g1, g2, g3) order
          std::vector<int64_t> perm;
          for (auto d : g1) perm.push_back(d);
          for (auto d : g2) perm.push_back(d);
          for (auto d : g3) perm.push_back(d);
          TView pv = v;
          std::vector<int64_t> pshape;
          for (size_t i = 0; i < perm.size(); ++i) {
            pv.shape[i] = v.shape[perm[i]];
            pv.stride[i] = v.stride[perm[i]];
            pshape.push_back(v.shape[perm[i]]);
          }
          TView m = materialize(pv, pshape, xn.dt);
          std::vector<int64_t> q1, q2, q3;
          int k = 0;
          for (size_t i = 0; i < g1.size(); ++i) q1.push_back(k++);
          for (size_t i = 0; i < g2.size(); ++i) q2.push_back(k++);
          for (size_t i = 0; i < g3.size(); ++i) q3.push_back(k++);
          collapse(m, q1, z[0], s[0]);
          collapse(m, q2, z[1], s[1]);
          collapse(m, q3, z[2], s[2]);
          return m;
        }
        return v;
      };
      int64_t as[3], az[3], bs[3], bz[3];
      TView av = canon(n.in[0], lb, lf, lc, as, az);  // batch, M, K
      TView bv = canon(n.in[1], rb, rc, rf, bs, bz);  // batch, K, N
      if (az[0] != bz[0] || az[2] != bz[1]) fail(E_INVALID, "dot_general dimension mismatch in %" + n.name);
      GemmParams G{};
      G.a = av.p;
      G.b = bv.p;
      G.c = slot_ptr(oslot);
      G.a_dt = av.dt;
      G.b_dt = bv.dt;
      G.c_dt = kdt(n.dt);
      G.batch = az[0];
      G.M = az[1];
      G.K = az[2];
      G.N = bz[2];
      G.a_sb = as[0]; G.a_sm = as[1]; G.a_sk = as[2];
      G.b_sb = bs[0]; G.b_sk = bs[1]; G.b_sn = bs[2];
      G.c_sb = G.M * G.N;
      if (!(G.a_dt == KDT_F32 || G.a_dt == KDT_BF16 || G.a_dt == KDT_F16) ||
          !(G.b_dt == KDT_F32 || G.b_dt == KDT_BF16 || G.b_dt == KDT_F16) ||
          !(G.c_dt == KDT_F32 || G.c_dt == KDT_BF16 || G.c_dt == KDT_F16))
        fail(E_UNIMPLEMENTED, "dot_general on integer operands");
      *bytes_out = a.numel() * (int64_t)dt_size(a.dt) + b.numel() * (int64_t)dt_size(b.dt) +
                   n.numel() * (int64_t)dt_size(n.dt);
      *flops_out = 2 * G.batch * G.M * G.N * G.K;
      return G;
    }
  }
}

void Planner::emit_outputs() {
  std::vector<char> claimed_done(g_.nodes.size(), 0);
  for (int k = 0; k < O_; ++k) {
    int n = g_.outputs[k];
    const Node& nd = g_.nodes[n];
    int oslot = P_ + k;
    if (out_claim_[n] == k) continue;  // written in place by its producer
    TView dst = dense_view(oslot, nd.dt, nd.shape);
    if (is_splat(n)) {
      EwParams E{};
      E.rank = nd.rank();
      E.n = nd.numel();
      for (int d = 0; d < E.rank; ++d) E.dims[d] = nd.shape[d];
      EwInstr I{};
      I.op = EW_IMM;
      I.dt = (uint8_t)kdt(nd.dt);
      I.fimm = (float)loc_[n].splat;
      I.iimm = (int32_t)(int64_t)loc_[n].splat;
      E.code[0] = I;
      E.ncode = 1;
      E.out[0].p = dst.p;
      E.out[0].dt = kdt(nd.dt);
      E.out[0].reg = 0;
      E.nout = 1;
      push(K_EW, blob_of(E), "out." + nd.name, nd.numel() * (int64_t)dt_size(nd.dt));
      continue;
    }
    CopyParams C{};
    C.src = view_of(n);
    C.dst = dst;
    C.n = nd.numel();
    push(K_COPY, blob_of(C), "out." + nd.name, 2 * C.n * (int64_t)dt_size(nd.dt));
  }
}

void Planner::emit_unit(int u) {
  const Node& n = g_.nodes[u];
  if (pre_emitted_.count(u)) return;
  emitted_units_.insert(u);
  if (loc_[u].kind == Loc::ROW) {
    emit_row_region(region_of_[u]);
    return;
  }
  if (loc_[u].kind == Loc::EW) {
    std::vector<int> members;
    for (size_t i = 0; i < g_.nodes.size(); ++i)
      if (live_[i] && loc_[i].kind == Loc::EW && find((int)i) == u) members.push_back((int)i);
    std::sort(members.begin(), members.end());
    emit_ew_group(members);
    plan_.n_fused_groups++;
    return;
  }
  (void)n;
  emit_node_kernel(u);
}

void Planner::emit_all() {
  const int N = (int)g_.nodes.size();
  // unit of every kernel-producing node
  std::vector<int> unit(N, -1);
  for (int i = 0; i < N; ++i) {
    if (!live_[i]) continue;
    if (loc_[i].kind == Loc::EW) unit[i] = find(i);
    else if (loc_[i].kind == Loc::ROW) unit[i] = regions_[region_of_[i]].root;
    else if (loc_[i].kind == Loc::BUF && g_.nodes[i].op != Op::Param && g_.nodes[i].op != Op::Constant) unit[i] = i;
  }
  std::map<int, std::set<int>> deps, rdeps;
  std::set<int> units;
  for (int i = 0; i < N; ++i) {
    if (unit[i] < 0) continue;
    units.insert(unit[i]);
    for (int o : ins_[i]) {
      if (is_splat(o)) continue;
      int r = view_root(o);
      if (unit[r] >= 0 && unit[r] != unit[i]) {
        deps[unit[i]].insert(unit[r]);
        rdeps[unit[r]].insert(unit[i]);
      }
    }
  }
  std::map<int, int> indeg;
  std::map<int, int> umin;
  for (int i = 0; i < N; ++i)
    if (unit[i] >= 0 && !umin.count(unit[i])) umin[unit[i]] = i;
  std::priority_queue<std::pair<int, int>, std::vector<std::pair<int, int>>, std::greater<>> q;
  for (int u : units) {
    indeg[u] = (int)deps[u].size();
    if (indeg[u] == 0) q.push({umin[u], u});
  }
  size_t done = 0;
  while (!q.empty()) {
    int u = q.top().second;
    q.pop();
    emit_unit(u);
    done++;
    for (int v : rdeps[u])
      if (--indeg[v] == 0) q.push({umin[v], v});
  }
  if (done != units.size()) fail(E_INTERNAL, "planner produced a cyclic schedule");
}

void Planner::allocate_arena() {
  // greedy interval allocation, first fit over active blocks sorted by offset
  const int T = (int)tmp_bytes_.size();
  std::vector<int> order(T);
  for (int i = 0; i < T; ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](int a, int b) {
    return tmp_first_[a] != tmp_first_[b] ? tmp_first_[a] < tmp_first_[b] : a < b;
  });
  std::vector<int64_t> off(T, 0);
  // buffers under 1 MiB get memory of their own (a decode step's temporaries
  // total a few MB): no two of them ever share bytes, so the scheduler sees
  // only true data dependencies between the small kernels that use them
  int64_t small_end = 0;
  for (int b : order) {
    if (tmp_bytes_[b] >= (1 << 20)) continue;
    off[b] = small_end;
    small_end += (tmp_bytes_[b] + 255) & ~int64_t(255);
  }
  std::multimap<int64_t, int> active;  // offset -> buffer (large buffers, reused after the small region)
  int64_t peak = small_end;
  for (int b : order) {
    if (tmp_bytes_[b] < (1 << 20)) continue;
    for (auto it = active.begin(); it != active.end();) {
      if (tmp_last_[it->second] < tmp_first_[b]) it = active.erase(it);
      else ++it;
    }
    int64_t sz = (tmp_bytes_[b] + 255) & ~int64_t(255);
    int64_t cand = small_end;
    for (auto& kv : active) {
      int64_t s = kv.first, e = kv.first + ((tmp_bytes_[kv.second] + 255) & ~int64_t(255));
      if (cand + sz <= s) break;
      cand = std::max(cand, e);
    }
    off[b] = cand;
    active.insert({cand, b});
    peak = std::max(peak, cand + sz);
  }
  plan_.arena_bytes = peak;
  plan_.tmp_offsets = off;
  plan_.tmp_bytes = tmp_bytes_;
}

void Planner::run() {
  const int N = (int)g_.nodes.size();
  P_ = (int)g_.params.size();
  O_ = (int)g_.outputs.size();
  plan_.name = g_.name;
  plan_.n_nodes = N;
  for (int p : g_.params) plan_.params.push_back({g_.nodes[p].dt, g_.nodes[p].shape});
  for (int o : g_.outputs) plan_.outs.push_back({g_.nodes[o].dt, g_.nodes[o].shape});
  plan_.out_alias_param.assign(O_, -1);
  ins_.assign(N, {});
  for (int i = 0; i < N; ++i) ins_[i] = g_.nodes[i].in;
  auto liveness = [&]() {
    users_.assign(N, {});
    for (int i = 0; i < N; ++i)
      for (int x : ins_[i]) users_[x].push_back(i);
    live_.assign(N, 0);
    std::vector<int> stack(g_.outputs.begin(), g_.outputs.end());
    while (!stack.empty()) {
      int x = stack.back();
      stack.pop_back();
      if (live_[x]) continue;
      live_[x] = 1;
      for (int y : ins_[x]) stack.push_back(y);
    }
  };
  liveness();
  for (int i = 0; i < N; ++i)
    if (live_[i] && g_.nodes[i].op == Op::NanCheck)
      fail(E_UNIMPLEMENTED, "custom_call " + std::string(g_.nodes[i].i0 ? "check_non_inf" : "check_non_nan") +
                                ": its result is used by the graph; the assertion is not executed on the device");
  if (opt_.fast_kernels) {
    // fused attention: the matched block's interior disappears, the probs.V
    // dot becomes one kernel reading q, the K/V caches and the mask
    for (AttnMatch& am : match_attention(g_, live_, users_)) {
      // a mask of the printed causal / sliding-window form is computed in the
      // kernel from the position: its chain (or literal) leaves the plan
      MaskForm mf;
      if (!getenv_off("CLJXLA_B200_MASK_FORM") &&
          match_mask_form(g_, am.mask, g_.nodes[am.d2].shape[2], g_.nodes[am.kc].shape[2], mf)) {
        mask_form_[am.d2] = mf;
        ins_[am.d2] = {am.q, am.kc, am.vc};
        if (mf.pos_param >= 0) ins_[am.d2].push_back(mf.pos_param);
      } else {
        ins_[am.d2] = {am.q, am.kc, am.vc, am.mask};
      }
      attn_[am.d2] = am;
    }
    if (!attn_.empty()) liveness();
    // greedy sampling: the printed argmax (tensor.clj:519-532) becomes one kernel
    for (int i = 0; i < N; ++i) {
      if (!live_[i]) continue;
      const int x = match_argmax(i);
      if (x < 0) continue;
      ins_[i] = {x};
      argmax_[i] = x;
    }
    if (!argmax_.empty()) liveness();
  }
  {
    // a dynamic_update_slice whose update is a float->float convert reads the
    // unconverted value and rounds it while storing (the KV-cache write of a
    // RoPE result computed in f32, attention.clj:108 + :135-168)
    bool rewired = false;
    for (int i = 0; i < N; ++i) {
      const Node& d = g_.nodes[i];
      if (!live_[i] || d.op != Op::DUS) continue;
      const int u = ins_[i][1];
      const Node& un = g_.nodes[u];
      if (un.op != Op::Convert || !dt_is_float(un.dt) || !dt_is_float(g_.nodes[un.in[0]].dt) ||
          g_.nodes[un.in[0]].shape != un.shape)
        continue;
      int live_users = 0;
      for (int x : users_[u]) live_users += live_[x] ? 1 : 0;
      bool returned = false;
      for (int o : g_.outputs) returned |= o == u;
      if (live_users != 1 || returned) continue;
      ins_[i][1] = un.in[0];
      rewired = true;
    }
    if (rewired) liveness();
  }
  for (int i = 0; i < N; ++i) plan_.n_live += live_[i];
  mat_slot_.assign(N, -1);
  out_claim_.assign(N, -1);
  if (opt_.kv_in_place) {
    // KV-cache updates returned as results: run them in place over the
    // argument's storage (the runtime versions the argument, see runtime.h)
    for (int k = 0; k < O_; ++k) {
      int n = g_.outputs[k];
      const Node& nd = g_.nodes[n];
      if (nd.op != Op::DUS || inplace_of_.count(n) || nd.rank() > CLJXLA_MAXR) continue;
      int p = nd.in[0];
      if (g_.nodes[p].op != Op::Param || g_.nodes[p].dt != nd.dt) continue;
      int live_users = 0;
      for (int u : users_[p]) live_users += live_[u] ? 1 : 0;
      bool returned = false;
      for (int o : g_.outputs) returned |= o == p;
      if (live_users != 1 || returned) continue;
      int pidx = -1;
      for (int q = 0; q < P_; ++q)
        if (g_.params[q] == p) pidx = q;
      bool taken = false;
      for (auto& d : plan_.inplace) taken |= d.param == pidx;
      if (pidx < 0 || taken) continue;
      const Node& up = g_.nodes[nd.in[1]];
      InplaceDus d;
      d.out = k;
      d.param = pidx;
      d.rank = nd.rank();
      d.dt = nd.dt;
      for (int i = 0; i < d.rank; ++i) {
        d.out_shape[i] = nd.shape[i];
        d.upd_shape[i] = up.shape[i];
      }
      d.undo_bytes = 8 * CLJXLA_MAXR + up.numel() * (int64_t)dt_size(nd.dt);
      d.undo_slot = P_ + O_ + (int)plan_.inplace.size();
      inplace_of_[n] = (int)plan_.inplace.size();
      plan_.inplace.push_back(d);
      plan_.out_alias_param[k] = pidx;
    }
    U_ = (int)plan_.inplace.size();
  }
  classify();
  build_row_regions();
  // outputs produced by a kernel are written straight into the result buffer
  for (int k = 0; k < O_; ++k) {
    int n = g_.outputs[k];
    if (out_claim_[n] >= 0) continue;
    if ((loc_[n].kind == Loc::BUF && g_.nodes[n].op != Op::Param && g_.nodes[n].op != Op::Constant &&
         g_.nodes[n].op != Op::AllReduce) ||  // a collective's result stays in the arena (graph capture)
        loc_[n].kind == Loc::EW || loc_[n].kind == Loc::ROW)
      out_claim_[n] = k;
  }
  group_elementwise();
  decide_materialisation();
  emit_all();
  emit_outputs();
  allocate_arena();
  // tensor maps and the status word sit in the table after the scratch slots
  for (Launch& l : plan_.launches) {
    if (l.kind != K_GEMM_TC) continue;
    TcGemmParams& t = *(TcGemmParams*)l.blob.data();
    // B copied before the dependency wait (CLJXLA_B200_TC_EARLY_B=1): a
    // parameter (a weight) that no launch writes (in-place KV updates write
    // their parameters).  Off by default: measured slower (Gemma-2-2B batch-32
    // decode 4.29 against 4.17 ms per step, Gemma-3-4B prefill 44.8 against
    // 44.2 ms), the early copies competing with the predecessor's traffic.
    const char* eb = getenv("CLJXLA_B200_TC_EARLY_B");
    t.b_const = eb && eb[0] == '1' && t.b.slot >= 0 && t.b.slot < (int)plan_.params.size() ? 1 : 0;
    for (const InplaceDus& ip : plan_.inplace)
      if (ip.param == t.b.slot) t.b_const = 0;
    const int slot = plan_.tmap_slot();
    t.tmap_a = DPtr{slot, 0, 128LL * t.tmap_a_index};
    t.tmap_b = DPtr{slot, 0, 128LL * t.tmap_b_index};
    t.status = DPtr{slot, 0, 128LL * (int64_t)plan_.tmaps.size()};
  }
  for (Launch& l : plan_.launches) {
    if (l.kind != K_ATTN_DECODE) continue;
    AttnParams& a = *(AttnParams*)l.blob.data();
    if (a.use_tc != 3) continue;
    plan_.needs_status = true;
    a.status = DPtr{plan_.tmap_slot(), 0, 128LL * (int64_t)plan_.tmaps.size()};
    a.has_status = 1;
  }
  for (Launch& l : plan_.launches) {
    if (l.kind != K_GEMV) continue;
    GemvParams& g = *(GemvParams*)l.blob.data();
    plan_.needs_status = true;
    g.status = DPtr{plan_.tmap_slot(), 0, 128LL * (int64_t)plan_.tmaps.size()};
    g.has_status = 1;
  }
  verify_plan(plan_);
  if (opt_.fuse) {
    schedule_and_merge(plan_);
    if (opt_.fast_kernels) {
      fuse_gemv_epilogues(plan_);
      fuse_row_epilogues(plan_);
      fuse_gemv_group_tails(plan_);
      link_gemv_prefetch(plan_);
      link_attention_hints(plan_);
      fuse_gemv_tails(plan_);
    }
    verify_plan(plan_);
  }
  if (const char* path = getenv("CLJXLA_B200_DUMP_PLAN")) {
    if (FILE* f = fopen(path, "a")) {
      fprintf(f, "# plan %s: %zu launches, arena %lld bytes\n", plan_.name.c_str(), plan_.launches.size(),
              (long long)plan_.arena_bytes);
      for (const Launch& l : plan_.launches)
        fprintf(f, "%s\t%lld\t%s\n", kernel_kind_name(l.kind), (long long)l.algo_bytes, l.label.c_str());
      fclose(f);
    }
  }
}

}  // namespace

std::unique_ptr<Plan> build_plan(const Graph& g, const PlanOptions& opt) {
  auto plan = std::make_unique<Plan>();
  if (opt.fuse) {
    int merged = 0;
    auto g2 = cse_graph(g, &merged);
    Planner p(*g2, opt, *plan);
    p.run();
    plan->n_nodes = (int)g.nodes.size();
    return plan;
  }
  Planner p(g, opt, *plan);
  p.run();
  return plan;
}

}  // namespace cljxla
