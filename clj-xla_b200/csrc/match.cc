// Structural matchers for fused kernels.
//
// The attention matcher recognises the block that gqa-causal-attention
// (attention.clj:287-375) and causal-self-attention (:227-285) print:
//
//   d1  = dot_general(q, K')             batch [0,1], contract [3]x[3]
//   ... = <elementwise chain on d1: multiply by the scale, optional
//          c*tanh(x/c) softcap, printer-inserted converts>
//   m   = add(chain, mask')              (either operand order)
//   sub = subtract(m, broadcast(reshape(reduce_max(m, dims [3]))))
//   e   = exponential(sub)
//   div = divide(e, broadcast(reshape(reduce_add(e, dims [3]))))
//   d2  = dot_general(div, V')           batch [0,1], contract [3]x[2]
//
// where K' / V' are either the caches themselves or the GQA form
// reshape(broadcast_in_dim(cache, [0,1,3,4])).  Every interior value must have
// no other consumer, so replacing the block by one kernel is exact.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <set>

#include "fast_kernels.h"

namespace cljxla {
namespace {

struct M {
  const Graph& g;
  const std::vector<char>& live;
  const std::vector<std::vector<int>>& users;
  const Node& N(int i) const { return g.nodes[i]; }
  int nuse(int i) const {
    int c = 0;
    for (int u : users[i]) c += live[u] ? 1 : 0;
    return c;
  }
  bool is_view(int i) const {
    const Node& n = N(i);
    return n.op == Op::Reshape || n.op == Op::Broadcast || n.op == Op::Transpose || n.op == Op::Slice ||
           (n.op == Op::Convert && N(n.in[0]).dt == n.dt);
  }
  bool splat(int i, double& v) const {
    const Node& n = N(i);
    if (n.op == Op::Constant) {
      if (!n.splat) return false;
      v = n.splat_val;
      return true;
    }
    if (is_view(i)) return splat(n.in[0], v);
    if (n.op == Op::Convert && splat(n.in[0], v)) {
      if (n.dt == DT::BF16) v = (double)bf16_to_f32(f32_to_bf16((float)v));
      else if (n.dt == DT::F16) v = (double)f16_to_f32(f32_to_f16((float)v));
      else if (n.dt == DT::F32) v = (double)(float)v;
      else return false;
      return true;
    }
    return false;
  }
  // broadcast(reshape(reduce(x, dims [rank-1]))) of kind k; returns the reduce node
  int row_reduce_bcast(int b, int kind, std::vector<int>& path) const {
    if (N(b).op != Op::Broadcast) return -1;
    int r = N(b).in[0];
    if (N(r).op != Op::Reshape) return -1;
    int red = N(r).in[0];
    const Node& R = N(red);
    if (R.op != Op::Reduce || R.i0 != kind || R.ia.size() != 1) return -1;
    const Node& in = N(R.in[0]);
    if (R.ia[0] != in.rank() - 1) return -1;
    const Node& Bn = N(b);
    for (size_t i = 0; i < Bn.ia.size(); ++i)
      if (Bn.ia[i] != (int64_t)i) return -1;
    if (nuse(b) != 1 || nuse(r) != 1 || nuse(red) != 1) return -1;
    path.push_back(b);
    path.push_back(r);
    path.push_back(red);
    return red;
  }
  // GQA form or direct cache: returns the cache node, appends absorbed views
  int kv_source(int x, int64_t nq, int& group, std::vector<int>& path) const {
    const Node& n = N(x);
    if (n.rank() != 4) return -1;
    if (n.op == Op::Reshape) {
      int b = n.in[0];
      const Node& Bn = N(b);
      if (Bn.op == Op::Broadcast && Bn.rank() == 5 && Bn.ia == std::vector<int64_t>{0, 1, 3, 4}) {
        const Node& c = N(Bn.in[0]);
        if (c.rank() != 4 || Bn.shape[1] != c.shape[1] || Bn.shape[3] != c.shape[2] || Bn.shape[4] != c.shape[3])
          return -1;
        if (n.shape[1] != Bn.shape[1] * Bn.shape[2] || n.shape[1] != nq) return -1;
        if (nuse(x) != 1 || nuse(b) != 1) return -1;
        group = (int)Bn.shape[2];
        path.push_back(x);
        path.push_back(b);
        return Bn.in[0];
      }
    }
    if (n.shape[1] != nq) return -1;
    group = 1;
    return x;
  }
};

bool dims_eq(const std::vector<int64_t>& a, std::initializer_list<int64_t> b) {
  return a == std::vector<int64_t>(b);
}

}  // namespace

std::vector<AttnMatch> match_attention(const Graph& g, const std::vector<char>& live,
                                       const std::vector<std::vector<int>>& users) {
  M m{g, live, users};
  std::vector<AttnMatch> out;
  std::set<int> taken;
  for (int d2 = 0; d2 < (int)g.nodes.size(); ++d2) {
    if (!live[d2]) continue;
    const Node& D2 = g.nodes[d2];
    if (D2.op != Op::Dot || D2.rank() != 4) continue;
    if (!dims_eq(D2.ia, {0, 1}) || !dims_eq(D2.ib, {0, 1}) || !dims_eq(D2.ic, {3}) || !dims_eq(D2.id, {2})) continue;
    AttnMatch am;
    am.d2 = d2;
    std::vector<int> ab;
    int div = D2.in[0];
    if (m.N(div).op != Op::Div || m.nuse(div) != 1) continue;
    int e = m.N(div).in[0];
    if (m.N(e).op != Op::Exp || m.nuse(e) != 2) continue;
    std::vector<int> path;
    int rsum = m.row_reduce_bcast(m.N(div).in[1], RED_ADD, path);
    double z;
    if (rsum < 0 || m.N(rsum).in[0] != e || !m.splat(m.N(rsum).in[1], z) || z != 0.0) continue;
    int sub = m.N(e).in[0];
    if (m.N(sub).op != Op::Sub || m.nuse(sub) != 1) continue;
    int mm = m.N(sub).in[0];
    int rmax = m.row_reduce_bcast(m.N(sub).in[1], RED_MAX, path);
    if (rmax < 0 || m.N(rmax).in[0] != mm || !m.splat(m.N(rmax).in[1], z) || z > -1e20) continue;
    if (m.N(mm).op != Op::Add || m.nuse(mm) != 2) continue;
    // walk each operand of the add back to a q.K^T dot through the score chain
    int d1 = -1, mask = -1;
    std::vector<int> chain;
    for (int side = 0; side < 2 && d1 < 0; ++side) {
      std::vector<int> ch;
      int c = m.N(mm).in[side];
      bool ok = true;
      while (ok) {
        const Node& C = m.N(c);
        if (C.op == Op::Dot) break;
        if (m.nuse(c) != 1) { ok = false; break; }
        if (!(C.op == Op::Mul || C.op == Op::Div || C.op == Op::Add || C.op == Op::Sub || C.op == Op::Tanh ||
              C.op == Op::Convert || C.op == Op::Neg || C.op == Op::Max || C.op == Op::Min)) { ok = false; break; }
        if (!dt_is_float(C.dt)) { ok = false; break; }
        int pred = -1;
        for (int o : C.in) {
          double v;
          if (m.splat(o, v)) continue;
          if (pred >= 0) { ok = false; break; }
          pred = o;
        }
        if (!ok || pred < 0) { ok = false; break; }
        ch.push_back(c);
        if (ch.size() > 8) { ok = false; break; }
        c = pred;
      }
      if (!ok) continue;
      const Node& D1 = m.N(c);
      if (D1.op != Op::Dot || D1.rank() != 4 || m.nuse(c) != 1) continue;
      if (!dims_eq(D1.ia, {0, 1}) || !dims_eq(D1.ib, {0, 1}) || !dims_eq(D1.ic, {3}) || !dims_eq(D1.id, {3})) continue;
      d1 = c;
      std::reverse(ch.begin(), ch.end());
      chain = ch;
      mask = m.N(mm).in[1 - side];
    }
    if (d1 < 0) continue;
    const Node& D1 = m.N(d1);
    const Node& Q = m.N(D1.in[0]);
    int64_t B = Q.shape[0], nq = Q.shape[1], Sq = Q.shape[2], hd = Q.shape[3];
    int gk = 1, gv = 1;
    int kc = m.kv_source(D1.in[1], nq, gk, path);
    int vc = m.kv_source(D2.in[1], nq, gv, path);
    if (kc < 0 || vc < 0 || gk != gv) continue;
    const Node& K = m.N(kc);
    const Node& V = m.N(vc);
    int64_t T = K.shape[2];
    if (K.shape[0] != B || V.shape != K.shape || K.shape[3] != hd || nq % K.shape[1] != 0 ||
        nq / K.shape[1] != gk)
      continue;
    if (!(hd == 32 || hd == 64 || hd == 128 || hd == 256)) continue;
    if (!(K.dt == DT::BF16 || K.dt == DT::F32) || V.dt != K.dt) continue;
    const Node& Mn = m.N(mm);
    if (Mn.shape != std::vector<int64_t>{B, nq, Sq, T} || m.N(mask).shape != Mn.shape) continue;
    if (D2.shape != std::vector<int64_t>{B, nq, Sq, hd}) continue;
    if (!(D2.dt == DT::F32 || D2.dt == DT::BF16)) continue;
    am.d1 = d1;
    am.q = D1.in[0];
    am.kc = kc;
    am.vc = vc;
    am.mask = mask;
    am.m = mm;
    am.sub = sub;
    am.exp = e;
    am.div = div;
    am.chain = chain;
    am.group = gk;
    ab = path;
    ab.push_back(d1);
    for (int c : chain) ab.push_back(c);
    for (int x : {mm, sub, e, div}) ab.push_back(x);
    bool clash = false;
    for (int x : ab) clash |= taken.count(x) > 0;
    if (clash) continue;
    for (int x : ab) taken.insert(x);
    am.absorbed = ab;
    out.push_back(am);
  }
  return out;
}

// ---------------------------------------------------------------------------
// Mask forms.  generate-causal-mask (attention.clj:189-224) prints either a
// chain over iotas and the traced position,
//   d = j - (i + p);  m = select(d > 0, -1e4, 0);  [m = select(d < -W, -1e4, m)]
// viewed up to the attention's [B, nq, Sq, T] operand, or (numeric position,
// static sizes) the same values as a dense [1, 1, Sq, T] literal.  Both are
// recognised exactly: the chain by an affine analysis of d over the operand's
// coordinates, the literal by checking every element.
namespace {

struct Aff {
  std::vector<int64_t> coef;  // per axis of the node: value += coef[a] * coordinate a
  int64_t cp = 0;             // times the position
  int pparam = -1;            // graph parameter holding the position (element 0)
  int64_t c0 = 0;
  bool same(const Aff& o) const {
    return coef == o.coef && cp == o.cp && c0 == o.c0 && (cp == 0 || pparam == o.pparam);
  }
};

struct MaskAn {
  const Graph& g;
  const Node& N(int i) const { return g.nodes[i]; }
  static bool is_view(const Graph& g, int i) {
    const Node& n = g.nodes[i];
    return n.op == Op::Reshape || n.op == Op::Broadcast || n.op == Op::Transpose ||
           (n.op == Op::Convert && g.nodes[n.in[0]].dt == n.dt);
  }
  // a one-element constant (splat or dense), through views and exact converts
  bool scalar(int x, double& v) const {
    const Node& n = N(x);
    if (n.op == Op::Constant) {
      if (n.splat) { v = n.splat_val; return true; }
      if (n.numel() != 1) return false;
      switch (n.dt) {
        case DT::F32: { float f; memcpy(&f, n.data.data(), 4); v = f; return true; }
        case DT::I32: { int32_t i; memcpy(&i, n.data.data(), 4); v = i; return true; }
        case DT::F64: { memcpy(&v, n.data.data(), 8); return true; }
        default: return false;
      }
    }
    if (is_view(g, x) || n.op == Op::Slice) return scalar(n.in[0], v);
    if (n.op == Op::Convert && scalar(n.in[0], v)) {
      if (n.dt == DT::F32) return (double)(float)v == v;
      if (n.dt == DT::I32) return (double)(int32_t)v == v;
      return false;
    }
    return false;
  }
  // maps per-axis coefficients of a view's operand onto the view's axes
  bool view_map(int x, const std::vector<int64_t>& in, std::vector<int64_t>& out) const {
    const Node& n = N(x);
    const Node& src = N(n.in[0]);
    out.assign(n.rank(), 0);
    switch (n.op) {
      case Op::Convert: out = in; return true;
      case Op::Transpose:
        for (int a = 0; a < n.rank(); ++a) out[a] = in[n.ia[a]];
        return true;
      case Op::Broadcast:
        for (int a = 0; a < src.rank(); ++a) out[n.ia[a]] = src.shape[a] == 1 ? 0 : in[a];
        return true;
      case Op::Reshape: {
        std::vector<int> ai, ao;
        for (int a = 0; a < src.rank(); ++a) if (src.shape[a] != 1) ai.push_back(a);
        for (int a = 0; a < n.rank(); ++a) if (n.shape[a] != 1) ao.push_back(a);
        bool aligned = ai.size() == ao.size();
        for (size_t k = 0; aligned && k < ai.size(); ++k) aligned = src.shape[ai[k]] == n.shape[ao[k]];
        if (aligned) {
          for (size_t k = 0; k < ai.size(); ++k) out[ao[k]] = in[ai[k]];
          return true;
        }
        for (int a : ai) if (in[a] != 0) return false;  // merged / split axes of a varying value
        return true;
      }
      default: return false;
    }
  }
  bool aff(int x, Aff& a, int depth = 0) const {
    if (depth > 64) return false;
    const Node& n = N(x);
    a = Aff{};
    a.coef.assign(n.rank(), 0);
    double v;
    if (scalar(x, v)) {
      if (v != std::floor(v) || std::fabs(v) > (double)(1 << 23)) return false;
      a.c0 = (int64_t)v;
      return true;
    }
    switch (n.op) {
      case Op::Iota:
        if (n.i0 < 0 || n.i0 >= n.rank() || n.shape[n.i0] > (1 << 23)) return false;
        a.coef[n.i0] = 1;
        return true;
      case Op::Param:
        if (n.numel() != 1 || n.dt != DT::I32) return false;
        a.cp = 1;
        a.pparam = x;
        return true;
      case Op::Slice: {
        // element 0 of an i32 parameter (the first column of pos / pos_ids)
        const Node& src = N(n.in[0]);
        if (n.numel() != 1 || src.op != Op::Param || src.dt != DT::I32) return false;
        for (int64_t s0 : n.ia) if (s0 != 0) return false;
        a.cp = 1;
        a.pparam = n.in[0];
        return true;
      }
      case Op::Convert: {
        // integer values stay exact through i32 / f32 / f64 (|value| < 2^24)
        if (!(n.dt == DT::F32 || n.dt == DT::I32 || n.dt == DT::F64 || n.dt == DT::I64)) return false;
        const DT s = N(n.in[0]).dt;
        if (!(s == DT::F32 || s == DT::I32 || s == DT::F64 || s == DT::I64)) return false;
        return aff(n.in[0], a, depth + 1);
      }
      case Op::Reshape: case Op::Broadcast: case Op::Transpose: {
        Aff in;
        if (!aff(n.in[0], in, depth + 1)) return false;
        std::vector<int64_t> c;
        if (!view_map(x, in.coef, c)) return false;
        a = in;
        a.coef = c;
        return true;
      }
      case Op::Add: case Op::Sub: {
        Aff l, r;
        if (!aff(n.in[0], l, depth + 1) || !aff(n.in[1], r, depth + 1)) return false;
        if (l.coef.size() != r.coef.size()) return false;
        const int64_t sg = n.op == Op::Add ? 1 : -1;
        if (l.cp && r.cp && l.pparam != r.pparam) return false;
        a.coef = l.coef;
        for (size_t k = 0; k < a.coef.size(); ++k) a.coef[k] += sg * r.coef[k];
        a.cp = l.cp + sg * r.cp;
        a.pparam = a.cp ? (l.cp ? l.pparam : r.pparam) : -1;
        a.c0 = l.c0 + sg * r.c0;
        return true;
      }
      case Op::Neg: {
        if (!aff(n.in[0], a, depth + 1)) return false;
        for (auto& c : a.coef) c = -c;
        a.cp = -a.cp;
        a.c0 = -a.c0;
        return true;
      }
      default: return false;
    }
  }
  // value = mv where d > gt or d < lt, else z (d affine over the node's axes)
  struct Piece {
    Aff d;
    bool has_gt = false, has_lt = false, cst = false;
    int64_t gt = 0, lt = 0;
    double mv = 0, z = 0;
  };
  bool piece(int x, Piece& f, int depth = 0) const {
    if (depth > 8) return false;
    double v;
    if (scalar(x, v)) {
      f = Piece{};
      f.cst = true;
      f.z = v;
      return true;
    }
    const Node& n = N(x);
    if (n.op != Op::Select) return false;
    const Node& c = N(n.in[0]);
    double mv;
    if (c.op != Op::Compare || !scalar(n.in[1], mv)) return false;
    Piece inner;
    if (!piece(n.in[2], inner, depth + 1)) return false;
    int dir = (int)c.i0;
    double k;
    Aff d;
    if (scalar(c.in[1], k)) {
      if (!aff(c.in[0], d)) return false;
    } else if (scalar(c.in[0], k)) {  // constant on the left: mirror the direction
      if (!aff(c.in[1], d)) return false;
      dir = dir == CMP_GT ? CMP_LT : dir == CMP_LT ? CMP_GT : dir == CMP_GE ? CMP_LE : dir == CMP_LE ? CMP_GE : dir;
    } else {
      return false;
    }
    if (k != std::floor(k) || std::fabs(k) > (double)(1 << 23)) return false;
    if (d.coef.size() != (size_t)n.rank()) return false;
    if (inner.cst) {
      f = Piece{};
      f.d = d;
      f.z = inner.z;
    } else {
      if (!inner.d.same(d) || inner.mv != mv) return false;
      f = inner;
    }
    f.mv = mv;
    const int64_t ki = (int64_t)k;
    if (dir == CMP_GT || dir == CMP_GE) {
      if (f.has_gt) return false;
      f.has_gt = true;
      f.gt = dir == CMP_GT ? ki : ki - 1;
    } else if (dir == CMP_LT || dir == CMP_LE) {
      if (f.has_lt) return false;
      f.has_lt = true;
      f.lt = dir == CMP_LT ? ki : ki + 1;
    } else {
      return false;
    }
    return true;
  }
};

}  // namespace

bool match_mask_form(const Graph& g, int mask, int64_t Sq, int64_t T, MaskForm& f) {
  MaskAn an{g};
  const Node& M = g.nodes[mask];
  if (M.rank() != 4 || M.shape[2] != Sq || M.shape[3] != T || M.dt != DT::F32) return false;
  if (Sq >= (1 << 23) || T >= (1 << 23)) return false;
  // views from the operand down to the value that defines the mask
  std::vector<int> views;
  int base = mask;
  while (MaskAn::is_view(g, base)) {
    views.push_back(base);
    base = g.nodes[base].in[0];
    if (views.size() > 16) return false;
  }
  auto lift = [&](std::vector<int64_t> c, std::vector<int64_t>& out) {
    for (size_t k = views.size(); k-- > 0;) {
      std::vector<int64_t> o;
      if (!an.view_map(views[k], c, o)) return false;
      c.swap(o);
    }
    out = c;
    return true;
  };
  const Node& Bn = g.nodes[base];
  if (Bn.op == Op::Constant && !Bn.splat && Bn.dt == DT::F32) {
    // a literal (the printer emits it flat and reshapes it: the reshapes right
    // above it only reinterpret its row-major data); its last two axes must
    // become the operand's query and key axes
    std::vector<int64_t> lshape = Bn.shape;
    while (!views.empty() && g.nodes[views.back()].op == Op::Reshape) {
      lshape = g.nodes[views.back()].shape;
      views.pop_back();
    }
    const int r = (int)lshape.size();
    if (r < 2) return false;
    const int64_t ls = lshape[r - 2], lt = lshape[r - 1];
    if (Bn.numel() != ls * lt || lt != T || !(ls == Sq || Sq == 1)) return false;
    std::vector<int64_t> ei(r, 0), ej(r, 0), oi, oj;
    ei[r - 2] = 1;
    ej[r - 1] = 1;
    if (!lift(ei, oi) || !lift(ej, oj)) return false;
    if (oj != std::vector<int64_t>{0, 0, 0, 1}) return false;
    if (Sq > 1 && oi != std::vector<int64_t>{0, 0, 1, 0}) return false;
    if (ls != Sq) return false;
    const float* v = (const float*)Bn.data.data();
    float hi = -INFINITY, lo = INFINITY;
    for (int64_t e = 0; e < ls * lt; ++e) {
      if (!std::isfinite(v[e])) return false;
      hi = std::max(hi, v[e]);
      lo = std::min(lo, v[e]);
    }
    if (!(lo < hi)) return false;
    // unmasked (the larger value) positions must be exactly d = j - i in [dlo, dhi]
    int64_t dlo = INT64_MAX, dhi = INT64_MIN;
    for (int64_t i = 0; i < ls; ++i)
      for (int64_t j = 0; j < lt; ++j) {
        const float x = v[i * lt + j];
        if (x != hi && x != lo) return false;
        if (x == hi) { dlo = std::min(dlo, j - i); dhi = std::max(dhi, j - i); }
      }
    for (int64_t i = 0; i < ls; ++i)
      for (int64_t j = 0; j < lt; ++j)
        if ((v[i * lt + j] == hi) != (j - i >= dlo && j - i <= dhi)) return false;
    f = MaskForm{};
    f.off = 0;
    f.gt = dhi;
    f.has_lt = dlo > -(ls - 1);
    f.lt = f.has_lt ? dlo : 0;
    f.mv = lo;
    f.z = hi;
    return true;
  }
  MaskAn::Piece p;
  if (!an.piece(base, p) || p.cst || !p.has_gt) return false;
  std::vector<int64_t> c;
  if (!lift(p.d.coef, c)) return false;
  // d must be j - qi - pos + c0 over the operand's axes
  if (c[3] != 1 || c[0] != 0 || c[1] != 0) return false;
  if (Sq > 1 && c[2] != -1) return false;
  if (!(p.d.cp == -1 || p.d.cp == 0)) return false;
  if (std::fabs(p.mv) > 3.0e38 || std::fabs(p.z) > 3.0e38 || (double)(float)p.mv != p.mv || (double)(float)p.z != p.z)
    return false;
  f = MaskForm{};
  f.pos_param = p.d.cp ? p.d.pparam : -1;
  f.off = -p.d.c0;
  f.gt = p.gt;
  f.has_lt = p.has_lt;
  f.lt = p.lt;
  f.mv = (float)p.mv;
  f.z = (float)p.z;
  return std::llabs(f.off) < (1 << 23) && std::llabs(f.gt) < (1 << 23) && std::llabs(f.lt) < (1 << 23);
}

}  // namespace cljxla
