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

}  // namespace cljxla
