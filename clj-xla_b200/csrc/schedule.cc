// Launch scheduling and horizontal fusion.
//
// The planner emits launches in a topological order of the graph that
// interleaves independent chains (the q and k branches of a layer: norm,
// rotate-half, RoPE, cache write).  This pass re-levels the launch list by the
// memory each launch actually touches - the physical byte ranges of the
// scratch arena (so buffers that share arena memory at different times stay
// ordered), the read-only constant and tensor-map tables, and, conservatively,
// the caller's buffers as one space - and then merges neighbouring launches of
// the same level that are compiled fused kernels of the same launch shape into
// one launch whose CTA ranges run the individual programs.  Nothing that
// conflicts is ever reordered or merged.
#include <algorithm>

#include "fast_kernels.h"
#include "jit.h"

namespace cljxla {
namespace {

// Arguments, results and undo records are buffers the executor binds per run:
// each is its own space (SP_BUF + slot), accessed as a whole.  A result that a
// KV update writes in place is the storage of its argument, so it shares the
// argument's space; other arguments may share storage with each other but are
// only read, and fresh results and undo records alias nothing.
enum Space { SP_ARENA, SP_CONST, SP_TMAP, SP_ABS, SP_BUF };

struct Access {
  int space;
  int64_t lo, hi;  // bytes in that space (SP_BUF: the whole buffer)
  bool write;
};

struct Collector {
  const Plan& p;
  std::vector<Access>& out;
  void add(const DPtr& d, int64_t bytes, bool write) {
    if (bytes <= 0) return;
    const int P = (int)p.params.size(), O = (int)p.outs.size(), U = (int)p.inplace.size();
    Access a{};
    a.write = write;
    if (d.slot < 0) {
      a.space = SP_ABS;
      a.lo = d.off;
      a.hi = d.off + bytes;
    } else if (d.slot < P + O + U) {
      int slot = d.slot;
      for (const InplaceDus& ip : p.inplace)
        if (slot == P + ip.out) slot = ip.param;
      a.space = SP_BUF + slot;
      a.lo = 0;
      a.hi = 1;
    } else if (d.slot == p.const_slot()) {
      a.space = SP_CONST;
      a.lo = d.off;
      a.hi = d.off + bytes;
    } else if (d.slot >= p.tmp_slot0() && d.slot < p.tmp_slot0() + (int)p.tmp_offsets.size()) {
      a.space = SP_ARENA;
      a.lo = p.tmp_offsets[d.slot - p.tmp_slot0()] + d.off;
      a.hi = a.lo + bytes;
    } else {
      a.space = SP_TMAP;
      a.lo = d.off;
      a.hi = d.off + bytes;
    }
    out.push_back(a);
  }
  void view(const TView& v, bool write) {
    int64_t hi = 0;
    for (int i = 0; i < v.rank; ++i) {
      if (v.shape[i] == 0) return;
      hi += (v.shape[i] - 1) * v.stride[i];
    }
    add(v.p, (hi + 1) * (int64_t)dt_size((DT)v.dt), write);
  }
  void strided(const DPtr& d, int dt, std::initializer_list<std::pair<int64_t, int64_t>> dims, bool write) {
    int64_t hi = 0;
    for (auto& ds : dims) {
      if (ds.first == 0) return;
      hi += (ds.first - 1) * ds.second;
    }
    add(d, (hi + 1) * (int64_t)dt_size((DT)dt), write);
  }
  void ew_inputs(const EwIn* in, int nin, int rank, const int64_t* dims) {
    for (int i = 0; i < nin; ++i) {
      TView v{};
      v.p = in[i].p;
      v.dt = in[i].dt;
      v.rank = rank;
      for (int d = 0; d < rank; ++d) { v.shape[d] = dims[d]; v.stride[d] = in[i].stride[d]; }
      if (in[i].sel_dim >= 0) v.shape[in[i].sel_dim] = in[i].sel_hi - in[i].sel_lo;
      view(v, false);
    }
  }
};

// false: unknown launch kind (treated as a barrier)
bool accesses(const Plan& p, const Launch& l, std::vector<Access>& out) {
  Collector c{p, out};
  const void* b = l.blob.data();
  for (const Launch& e : l.epi)  // an epilogue program runs inside the launch
    if (!accesses(p, e, out)) return false;
  for (const Launch& e : l.gtail)  // and so do group-tail programs
    if (!accesses(p, e, out)) return false;
  if (l.kind == K_FUSED_DUS) {
    for (const Launch& part : l.parts)
      if (!accesses(p, part, out)) return false;
    return true;
  }
  switch (l.kind) {
    case K_EW: {
      const EwParams& e = *(const EwParams*)b;
      c.ew_inputs(e.in, e.nin, e.rank, e.dims);
      for (int o = 0; o < e.nout; ++o) c.add(e.out[o].p, e.n * (int64_t)dt_size((DT)e.out[o].dt), true);
      return true;
    }
    case K_ROWNORM: {
      const RowParams& r = *(const RowParams*)b;
      c.ew_inputs(r.in, r.nin, r.rank, r.dims);
      for (int o = 0; o < r.nout; ++o)
        c.add(r.out[o].p, (r.out[o].scalar ? r.rows : r.rows * r.C) * (int64_t)dt_size((DT)r.out[o].dt), true);
      return true;
    }
    case K_REDUCE: {
      const ReduceParams& r = *(const ReduceParams*)b;
      c.view(r.in, false);
      c.add(r.out, r.n_out * (int64_t)dt_size((DT)r.out_dt), true);
      return true;
    }
    case K_COPY: {
      const CopyParams& r = *(const CopyParams*)b;
      c.view(r.src, false);
      c.view(r.dst, true);
      return true;
    }
    case K_GATHER: {
      const GatherParams& g = *(const GatherParams*)b;
      c.strided(g.table, g.table_dt, {{g.rows_table, g.table_row_stride}, {g.row_len, 1}}, false);
      c.view(g.idx, false);
      c.add(g.out, g.n_rows * g.row_len * (int64_t)dt_size((DT)g.table_dt), true);
      return true;
    }
    case K_DUS: {
      const DusParams& d = *(const DusParams*)b;
      c.view(d.operand, false);
      c.view(d.update, false);
      c.add(d.out, d.n * (int64_t)dt_size((DT)d.dt), true);
      for (int i = 0; i < d.rank; ++i)
        if (d.start_is_ptr[i]) c.add(d.start_ptr[i], (int64_t)dt_size((DT)d.start_dt[i]), false);
      if (d.has_undo) c.add(d.undo, 1, true);
      return true;
    }
    case K_GEMM: {
      const GemmParams& g = *(const GemmParams*)b;
      c.strided(g.a, g.a_dt, {{g.batch, g.a_sb}, {g.M, g.a_sm}, {g.K, g.a_sk}}, false);
      c.strided(g.b, g.b_dt, {{g.batch, g.b_sb}, {g.K, g.b_sk}, {g.N, g.b_sn}}, false);
      c.add(g.c, g.batch * g.M * g.N * (int64_t)dt_size((DT)g.c_dt), true);
      return true;
    }
    case K_GEMV: case K_GEMV_FUSED: case K_GEMV_TAIL: {
      const GemvParams& g = *(const GemvParams*)b;
      if (l.kind == K_GEMV_TAIL) {
        for (const Launch& part : l.parts)
          if (!accesses(p, part, out)) return false;
        c.add(g.tail_ctr, 4, true);
      }
      if (!l.gtail.empty()) {
        int64_t groups = 0;
        for (const Launch& q : l.gtail)
          groups += ((const RowParams*)(q.kind == K_FUSED_DUS ? q.parts[0] : q).blob.data())->rows;
        c.add(g.tail_ctr, 4 * groups, true);
      }
      if (l.kind == K_GEMV_FUSED) {  // x is computed in shared memory by the producer's program
        if (l.parts.size() != 1 || !accesses(p, l.parts[0], out)) return false;
      } else {
        c.add(g.x, ((g.M - 1) * g.x_sm + g.K) * (int64_t)dt_size((DT)g.x_dt), false);
      }
      for (int i = 0; i < g.nseg; ++i) {
        const int64_t n = g.seg_end[i] - (i ? g.seg_end[i - 1] : 0);
        c.add(g.w[i], n * g.K * 2, false);
        c.add(g.y[i], g.M * n * (int64_t)dt_size((DT)g.y_dt[i]), true);
      }
      return true;
    }
    case K_ATTN_DECODE: case K_ATTN_COMBINE: {
      const AttnParams& a = *(const AttnParams*)b;
      const int64_t rows = (int64_t)a.B * a.nq * a.Sq;
      const int64_t part = attention_part_bytes(a);
      if (l.kind == K_ATTN_DECODE) {
        c.view(a.q, false);
        c.view(a.k, false);
        c.view(a.v, false);
        if (a.mask_mode) {
          if (a.has_mask_pos) c.add(a.mask_pos, 4, false);
        } else {
          c.view(a.mask, false);
        }
        if (a.splits > 1) c.add(a.part, part, true);
        if (a.splits == 1 || a.use_counters) c.add(a.out, rows * a.hd * (int64_t)dt_size((DT)a.out_dt), true);
        if (a.splits > 1 && a.use_counters)
          c.add(a.counters, 4LL * a.B * a.nkv * ((a.Sq + a.qtile - 1) / a.qtile), true);
      } else {
        c.add(a.part, part, false);
        c.add(a.out, rows * a.hd * (int64_t)dt_size((DT)a.out_dt), true);
      }
      return true;
    }
    case K_ARGMAX: {
      const ArgmaxParams& a = *(const ArgmaxParams*)b;
      c.view(a.in, false);
      c.add(a.out, a.rows * 4, true);
      if (a.ctas > 1) {
        c.add(a.part, argmax_part_bytes(a), true);
        c.add(a.counters, a.rows * 4, true);
      }
      return true;
    }
    case K_ALLREDUCE: {
      // a collective orders only against what touches its operand and result:
      // every rank plans the same graph, so every rank issues its collectives in
      // the same (re-levelled) order
      const AllReduceParams& a = *(const AllReduceParams*)b;
      const int64_t bytes = a.count * (int64_t)dt_size((DT)a.dt);
      c.add(a.src, bytes, false);
      c.add(a.dst, bytes, true);
      return true;
    }
    case K_GEMM_TC: {
      const TcGemmParams& t = *(const TcGemmParams*)b;
      c.add(t.a, ((int64_t)(t.a_parts * t.M - 1) * t.a_ld + t.K) * 2, false);
      c.add(t.b, ((int64_t)(t.N - 1) * t.b_ld + t.K) * 2, false);
      c.add(t.c, (int64_t)t.M * t.N * (int64_t)dt_size((DT)t.c_dt), true);
      c.add(t.tmap_a, 128, false);
      c.add(t.tmap_b, 128, false);
      c.add(t.status, 4, true);
      if (t.ksplit > 1) {
        c.add(t.part, (int64_t)t.ksplit * t.M * t.N * 4, true);
        c.add(t.counters, 4LL * ((t.M + 127) / 128) * ((t.N + t.bn - 1) / t.bn), true);
      }
      return true;
    }
  }
  return false;
}

bool conflict(const std::vector<Access>& a, const std::vector<Access>& b) {
  for (const Access& x : a)
    for (const Access& y : b) {
      if (!x.write && !y.write) continue;
      if (x.space == SP_ABS || y.space == SP_ABS) return true;
      if (x.space != y.space) continue;
      if (x.lo < y.hi && y.lo < x.hi) return true;
    }
  return false;
}

// launch shape a compiled kernel would use; kinds that are not compiled fused kernels: false
bool merge_key(const Launch& l, int* kind, int* block, int* cluster) {
  if (l.kind == K_FUSED_DUS) return merge_key(l.parts[0], kind, block, cluster);
  if (l.kind == K_EW) {
    *kind = K_EW;
    *block = 256;
    *cluster = 1;
    return ((const EwParams*)l.blob.data())->n > 0;
  }
  if (l.kind == K_ROWNORM) {
    const RowParams& r = *(const RowParams*)l.blob.data();
    if (r.rows == 0) return false;
    int64_t g;
    row_launch_shape(r, block, cluster, &g);
    *kind = K_ROWNORM;
    return true;
  }
  return false;
}

// A KV-window write (in-place dynamic_update_slice) whose update is exactly
// the dense output of an earlier fused elementwise group or row region moves
// into that program: the program stores the element into the cache window as
// well (after saving the old value to the undo record), and the DUS launch
// disappears.  Only when no launch in between touches what the write reads or
// writes, so that it may run at the producer's place.
void fuse_dus_into_producers(Plan& p) {
  std::vector<Launch>& L = p.launches;
  for (size_t i = 0; i < L.size(); ++i) {
    if (L[i].kind != K_DUS) continue;
    DusParams D;
    memcpy(&D, L[i].blob.data(), sizeof(D));
    auto fl = [](int t) { return t == KDT_F32 || t == KDT_BF16 || t == KDT_F16; };
    if (!D.in_place || D.rank < 1 || D.update.rank != D.rank || !(D.update.dt == D.dt || (fl(D.update.dt) && fl(D.dt))))
      continue;
    int64_t nu = 1;
    bool dense = true;
    for (int d = D.rank - 1; d >= 0; --d) {
      if (D.update.shape[d] != D.upd_shape[d]) dense = false;
      if (D.upd_shape[d] != 1 && D.update.stride[d] != nu) dense = false;
      nu *= D.upd_shape[d];
    }
    if (!dense || nu == 0) continue;
    std::vector<Access> ua;
    {
      Collector c{p, ua};
      c.add(D.update.p, nu * (int64_t)dt_size((DT)D.update.dt), false);
    }
    long j = -1;
    for (long k = (long)i - 1; k >= 0; --k) {
      std::vector<Access> a;
      if (!accesses(p, L[k], a)) break;
      if (conflict(a, ua)) {
        j = k;
        break;
      }
    }
    if (j < 0) continue;
    Launch& pro = L[j];
    const Launch& base = pro.kind == K_FUSED_DUS ? pro.parts[0] : pro;
    int out = -1;
    if (base.kind == K_EW) {
      const EwParams& e = *(const EwParams*)base.blob.data();
      if (e.n != nu) continue;
      for (int o = 0; o < e.nout; ++o)
        if (e.out[o].p.slot == D.update.p.slot && e.out[o].p.off == D.update.p.off && e.out[o].dt == D.update.dt) out = o;
    } else if (base.kind == K_ROWNORM) {
      const RowParams& r = *(const RowParams*)base.blob.data();
      if (r.rows * r.C != nu) continue;
      for (int o = 0; o < r.nout; ++o)
        if (!r.out[o].scalar && r.out[o].p.slot == D.update.p.slot && r.out[o].p.off == D.update.p.off &&
            r.out[o].dt == D.update.dt)
          out = o;
    } else {
      continue;
    }
    if (out < 0) continue;
    std::vector<Access> da;
    if (!accesses(p, L[i], da)) continue;
    bool movable = true;
    for (size_t k = (size_t)j + 1; k < i && movable; ++k) {
      std::vector<Access> a;
      movable = accesses(p, L[k], a) && !conflict(da, a);
    }
    if (!movable) continue;
    Launch f;
    if (pro.kind == K_FUSED_DUS) {
      f = std::move(pro);
    } else {
      f.kind = K_FUSED_DUS;
      f.label = pro.label;
      f.algo_bytes = pro.algo_bytes;
      f.parts.push_back(std::move(pro));
    }
    const size_t nb = f.blob.size();
    f.blob.resize(nb + 4);
    memcpy(f.blob.data() + nb, &out, 4);
    f.label += "+" + L[i].label;
    f.algo_bytes += L[i].algo_bytes;
    f.parts.push_back(std::move(L[i]));
    L[j] = std::move(f);
    L.erase(L.begin() + i);
    --i;
  }
}

// The producer of a GEMV's x moves into the GEMV as a prologue when it is a
// fused elementwise group or row region whose output is exactly x (dense
// [M, K], x's type), x fits in shared memory, and no launch between the two
// touches what the producer reads or writes (so the producer may run at the
// GEMV's place).
void fuse_gemv_prologues(Plan& p, bool ew_only, bool rows_only) {
  std::vector<Launch>& L = p.launches;
  for (size_t i = 0; i < L.size(); ++i) {
    if (L[i].kind != K_GEMV) continue;
    GemvParams G;
    memcpy(&G, L[i].blob.data(), sizeof(G));
    const int xes = (int)dt_size((DT)G.x_dt);
    // one row only: batched rows take the tensor-core GEMV, which has no prologue
    // (a fused batch-8 GEMV on the CUDA cores measured 0.78 TB/s against 2.4 TB/s)
    if (G.M != 1 || G.M * G.K * xes > 144 * 1024 || G.nseg < 1) continue;
    // the last earlier launch writing x
    std::vector<Access> xa;
    {
      Collector c{p, xa};
      c.add(G.x, G.M * G.K * xes, false);
    }
    long j = -1;
    std::vector<Access> acc_j;
    for (long k = (long)i - 1; k >= 0; --k) {
      std::vector<Access> a;
      if (!accesses(p, L[k], a)) break;
      if (conflict(a, xa)) {
        j = k;
        acc_j = std::move(a);
        break;
      }
    }
    static const bool dbg = getenv("CLJXLA_B200_DEBUG_FUSE") != nullptr;
    if (dbg) fprintf(stderr, "gemv %s x slot %d off %lld: producer %ld %s\n", L[i].label.c_str(), G.x.slot,
                     (long long)G.x.off, j, j >= 0 ? L[j].label.c_str() : "-");
    if (j < 0) continue;
    const Launch& pro = L[j];
    int out = -1, nbuf = 0;
    if (pro.kind == K_ROWNORM && !ew_only) {
      const RowParams& r = *(const RowParams*)pro.blob.data();
      if (r.rows != G.M || r.C != G.K) continue;
      for (int o = 0; o < r.nout; ++o)
        if (!r.out[o].scalar && r.out[o].p.slot == G.x.slot && r.out[o].p.off == G.x.off && r.out[o].dt == G.x_dt) out = o;
      nbuf = r.nin + r.nout;
    } else if (pro.kind == K_EW && !rows_only) {
      const EwParams& e = *(const EwParams*)pro.blob.data();
      if (e.n != G.M * G.K) continue;
      for (int o = 0; o < e.nout; ++o)
        if (e.out[o].p.slot == G.x.slot && e.out[o].p.off == G.x.off && e.out[o].dt == G.x_dt) out = o;
      nbuf = e.nin + e.nout;
    } else {
      continue;
    }
    if (out < 0 || nbuf + 2 * G.nseg > JIT_MAXBUF) continue;
    bool movable = true;
    for (size_t k = (size_t)j + 1; k < i && movable; ++k) {
      std::vector<Access> a;
      movable = accesses(p, L[k], a) && !conflict(acc_j, a);
    }
    if (!movable) continue;
    G.pro_out = out;
    Launch f;
    f.kind = K_GEMV_FUSED;
    f.blob.resize(sizeof(G));
    memcpy(f.blob.data(), &G, sizeof(G));
    f.label = pro.label + "+" + L[i].label;
    f.algo_bytes = pro.algo_bytes + L[i].algo_bytes;
    f.algo_flops = pro.algo_flops + L[i].algo_flops;
    f.parts.push_back(std::move(L[j]));
    L[i] = std::move(f);
    L.erase(L.begin() + j);
    --i;
  }
}

}  // namespace

void fuse_gemv_epilogues(Plan& p) {
  const char* env = getenv("CLJXLA_B200_GEMV_EPILOGUE");
  if (env && env[0] == '0') return;
  std::vector<Launch>& L = p.launches;
  for (size_t i = 0; i < L.size(); ++i) {
    Launch& gl = L[i];
    if ((gl.kind != K_GEMV && gl.kind != K_GEMV_FUSED) || !gl.epi.empty()) continue;
    const GemvParams& G = *(const GemvParams*)gl.blob.data();
    if (G.M != 1 || G.nseg > 2 || (G.nseg == 2 && G.seg_end[1] != 2 * G.seg_end[0])) continue;
    const int64_t F = G.nseg == 2 ? G.seg_end[0] : G.N;
    // the first later launch touching the GEMV's outputs
    std::vector<Access> ya;
    {
      Collector c{p, ya};
      for (int s = 0; s < G.nseg; ++s) c.add(G.y[s], F * (int64_t)dt_size((DT)G.y_dt[s]), true);
    }
    size_t k = i + 1;
    std::vector<Access> ak;
    for (; k < L.size(); ++k) {
      ak.clear();
      if (!accesses(p, L[k], ak)) break;
      if (conflict(ak, ya)) break;
    }
    if (k >= L.size() || L[k].kind != K_EW) continue;
    const EwParams& e = *(const EwParams*)L[k].blob.data();
    if (e.n != F || e.nout < 1) continue;
    // every input on a GEMV output reads it at the element's own index; nothing
    // else the program touches overlaps the GEMV's outputs
    int64_t dense[CLJXLA_MAXR];
    {
      int64_t st = 1;
      for (int d = e.rank - 1; d >= 0; --d) {
        dense[d] = st;
        st *= e.dims[d];
      }
    }
    bool ok = true;
    std::vector<Access> rest;
    Collector rc{p, rest};
    for (int j = 0; j < e.nin && ok; ++j) {
      const EwIn& in = e.in[j];
      int seg = -1;
      for (int s = 0; s < G.nseg; ++s)
        if (in.p.slot == G.y[s].slot && in.p.off == G.y[s].off) seg = s;
      if (seg < 0) {
        int64_t hi = 0;
        for (int d = 0; d < e.rank; ++d) hi += (e.dims[d] - 1) * in.stride[d];
        rc.add(in.p, (hi + 1) * (int64_t)dt_size((DT)in.dt), false);
        continue;
      }
      if (in.sel_dim >= 0 || in.dt != G.y_dt[seg]) ok = false;
      for (int d = 0; d < e.rank && ok; ++d)
        if (e.dims[d] > 1 && in.stride[d] != dense[d]) ok = false;
    }
    for (int o = 0; o < e.nout; ++o) rc.add(e.out[o].p, e.n * (int64_t)dt_size((DT)e.out[o].dt), true);
    if (!ok || conflict(rest, ya)) continue;
    // the program may run at the GEMV's place: no launch between touches what it does
    std::vector<Access> ae;
    if (!accesses(p, L[k], ae)) continue;
    bool movable = true;
    for (size_t m = i + 1; m < k && movable; ++m) {
      std::vector<Access> a;
      movable = accesses(p, L[m], a) && !conflict(ae, a);
    }
    if (!movable) continue;
    gl.label += "+" + L[k].label;
    gl.algo_bytes += L[k].algo_bytes;
    gl.algo_flops += L[k].algo_flops;
    gl.epi.push_back(std::move(L[k]));
    L.erase(L.begin() + (long)k);
  }
}

namespace {

// The elementwise program `e` reads the outputs of row program `r` only
// within the row of each element it computes (element i of e belongs to row
// i / C of r): dense leading dims, the last dim within one row (a slice or a
// concatenate operand of it, as RoPE's rotate_half reads it).  It reads no
// other output of `others`.
bool row_local(const Plan& p, const RowParams& r, const EwParams& e, const std::vector<const Launch*>& others) {
  if (e.n != r.rows * r.C || e.rank < 1 || e.dims[e.rank - 1] != r.C) return false;
  int64_t dense[CLJXLA_MAXR];
  {
    int64_t st = 1;
    for (int d = e.rank - 1; d >= 0; --d) {
      dense[d] = st;
      st *= e.dims[d];
    }
  }
  std::vector<Access> other_w;
  {
    for (const Launch* o : others) {
      std::vector<Access> a;
      if (!accesses(p, *o, a)) return false;
      for (const Access& x : a)
        if (x.write) other_w.push_back(x);
    }
  }
  for (int j = 0; j < e.nin; ++j) {
    const EwIn& in = e.in[j];
    int out = -1;
    int64_t base = 0;
    for (int o = 0; o < r.nout; ++o) {
      if (r.out[o].scalar || r.out[o].p.slot != in.p.slot || in.p.slot < 0) continue;
      const int64_t es = (int64_t)dt_size((DT)r.out[o].dt);
      const int64_t d = in.p.off - r.out[o].p.off;
      if (d >= 0 && d < r.rows * r.C * es && d % es == 0 && in.dt == r.out[o].dt) {
        out = o;
        base = d / es;
      }
    }
    std::vector<Access> ia;
    {
      Collector ic{p, ia};
      int64_t hi = 0;
      for (int d = 0; d < e.rank; ++d) hi += (e.dims[d] - 1) * in.stride[d];
      ic.add(in.p, (hi + 1) * (int64_t)dt_size((DT)in.dt), false);
    }
    if (conflict(ia, other_w)) return false;
    if (out < 0) {  // not an output of r: must not be one either (another slot, or outside r's outputs)
      std::vector<Access> rw;
      Collector rc{p, rw};
      for (int o = 0; o < r.nout; ++o)
        if (!r.out[o].scalar) rc.add(r.out[o].p, r.rows * r.C * (int64_t)dt_size((DT)r.out[o].dt), true);
      if (conflict(ia, rw)) return false;
      continue;
    }
    if (base >= r.C) return false;  // the view starts in the first row
    for (int d = 0; d + 1 < e.rank; ++d)
      if (e.dims[d] > 1 && in.stride[d] != dense[d]) return false;
    if (in.stride[e.rank - 1] != 1) return false;
    const int64_t len = in.sel_dim == e.rank - 1 ? in.sel_hi - in.sel_lo : e.dims[e.rank - 1];
    if (in.sel_dim >= 0 && in.sel_dim != e.rank - 1) return false;
    if (base + len > r.C) return false;
  }
  return true;
}

}  // namespace

void fuse_gemv_group_tails(Plan& p) {
  // opt-in (CLJXLA_B200_GEMV_GROUP_TAIL=1): on Gemma-3-4B decode the per-head
  // norms, RoPE and KV writes run by the q/k/v GEMV's completing CTAs took 2.45
  // ms / step against 2.27 ms as their own launch (13 CTAs of 512 threads
  // right after the GEMV): the completing CTAs are the GEMV's last ones, and a
  // CTA that completes several heads runs them one after another
  const char* env = getenv("CLJXLA_B200_GEMV_GROUP_TAIL");
  if (!env || env[0] != '1') return;
  std::vector<Launch>& L = p.launches;
  for (size_t i = 0; i + 1 < L.size(); ++i) {
    Launch& gl = L[i];
    if ((gl.kind != K_GEMV && gl.kind != K_GEMV_FUSED) || !gl.epi.empty() || !gl.gtail.empty()) continue;
    GemvParams G;
    memcpy(&G, gl.blob.data(), sizeof(G));
    if (G.M != 1) continue;
    Launch& nx = L[i + 1];
    std::vector<Launch> parts;
    if (nx.kind == K_MULTI) parts = nx.parts;
    else if (nx.kind == K_ROWNORM || nx.kind == K_FUSED_DUS) parts.push_back(nx);
    else continue;
    std::vector<Access> ga, yw;
    if (!accesses(p, gl, ga)) continue;
    {
      Collector c{p, yw};
      for (int s = 0; s < G.nseg; ++s)
        c.add(G.y[s], (G.seg_end[s] - (s ? G.seg_end[s - 1] : 0)) * (int64_t)dt_size((DT)G.y_dt[s]), true);
    }
    bool ok = parts.size() <= 6;
    int64_t groups = 0;
    for (const Launch& q : parts) {
      if (!ok) break;
      const Launch& qb = q.kind == K_FUSED_DUS ? q.parts[0] : q;
      if (qb.kind != K_ROWNORM || q.epi.size() > 1) { ok = false; break; }
      const RowParams& r = *(const RowParams*)qb.blob.data();
      int blk, cl;
      int64_t grid;
      row_launch_shape(r, &blk, &cl, &grid);
      if (cl != 1 || grid != r.rows || r.C > 12 * 256) { ok = false; break; }
      // one input is a whole GEMV segment read row by row, densely
      int seg = -1;
      int64_t dense[CLJXLA_MAXR];
      {
        int64_t st = 1;
        for (int d = r.rank - 1; d >= 0; --d) {
          dense[d] = st;
          st *= r.dims[d];
        }
      }
      for (int j = 0; j < r.nin; ++j) {
        const EwIn& in = r.in[j];
        int sj = -1;
        for (int k = 0; k < G.nseg; ++k)
          if (in.p.slot == G.y[k].slot && in.p.off == G.y[k].off) sj = k;
        std::vector<Access> ia;
        {
          Collector ic{p, ia};
          int64_t hi = 0;
          for (int d = 0; d < r.rank; ++d) hi += (r.dims[d] - 1) * in.stride[d];
          ic.add(in.p, (hi + 1) * (int64_t)dt_size((DT)in.dt), false);
        }
        if (sj < 0) {
          if (conflict(ia, yw)) ok = false;  // part of a GEMV output, not read as a whole segment
          continue;
        }
        if (seg >= 0 && seg != sj) ok = false;
        seg = sj;
        if (in.sel_dim >= 0 || in.dt != G.y_dt[sj] ||
            G.seg_end[sj] - (sj ? G.seg_end[sj - 1] : 0) != r.rows * r.C)
          ok = false;
        for (int d = 0; d < r.rank && ok; ++d)
          if (r.dims[d] > 1 && in.stride[d] != dense[d]) ok = false;
      }
      if (seg < 0) ok = false;
      // what the part (and its epilogue) writes is not something the GEMV touches
      std::vector<Access> qa;
      if (!ok || !accesses(p, q, qa)) { ok = false; break; }
      std::vector<Access> qw;
      for (const Access& x : qa)
        if (x.write) qw.push_back(x);
      if (conflict(qw, ga)) ok = false;
      // the epilogue reads no GEMV output directly
      for (const Launch& e : q.epi) {
        std::vector<Access> ea;
        if (!accesses(p, e, ea) || conflict(ea, yw)) ok = false;
      }
      groups += r.rows;
    }
    if (!ok || groups == 0 || groups > 64) continue;
    const size_t off = (p.const_blob.size() + 15) & ~size_t(15);
    p.const_blob.resize(off + 4 * (size_t)groups, 0);
    G.tail_ctr = DPtr{p.const_slot(), 0, (int64_t)off};
    memcpy(gl.blob.data(), &G, sizeof(G));
    gl.label += "+" + nx.label;
    gl.algo_bytes += nx.algo_bytes;
    gl.gtail = std::move(parts);
    L.erase(L.begin() + (long)(i + 1));
  }
}

void fuse_row_epilogues(Plan& p) {
  const char* env = getenv("CLJXLA_B200_ROW_EPILOGUE");
  if (env && env[0] == '0') return;
  std::vector<Launch>& L = p.launches;
  for (size_t i = 0; i + 1 < L.size(); ++i) {
    if (L[i].kind != K_MULTI) continue;
    Launch& nx = L[i + 1];
    // the next launch's programs, one at a time
    std::vector<Launch> next;
    if (nx.kind == K_MULTI) next = nx.parts;
    else if (nx.kind == K_EW || nx.kind == K_FUSED_DUS) next.push_back(nx);
    else continue;
    std::vector<Launch> keep;
    bool moved = false;
    for (Launch& q : next) {
      const Launch& qb = q.kind == K_FUSED_DUS ? q.parts[0] : q;
      bool done = false;
      if (qb.kind == K_EW) {
        const EwParams& e = *(const EwParams*)qb.blob.data();
        for (size_t k = 0; k < L[i].parts.size() && !done; ++k) {
          Launch& rp = L[i].parts[k];
          if (rp.kind != K_ROWNORM || !rp.epi.empty()) continue;
          const RowParams& r = *(const RowParams*)rp.blob.data();
          int blk, cl;
          int64_t grid;
          row_launch_shape(r, &blk, &cl, &grid);
          if (cl != 1 || grid != r.rows) continue;
          std::vector<const Launch*> others;
          for (size_t o = 0; o < L[i].parts.size(); ++o)
            if (o != k) others.push_back(&L[i].parts[o]);
          if (!row_local(p, r, e, others)) continue;
          // what the program writes is touched by no other part of the launch
          std::vector<Access> qa, oa;
          if (!accesses(p, q, qa)) continue;
          bool clash = false;
          for (const Launch* o : others) {
            oa.clear();
            if (!accesses(p, *o, oa) || conflict(qa, oa)) clash = true;
          }
          if (clash) continue;
          L[i].algo_bytes += q.algo_bytes;
          L[i].label += "+" + q.label;
          rp.label += "+" + q.label;
          rp.epi.push_back(q);
          done = moved = true;
        }
      }
      if (!done) keep.push_back(std::move(q));
    }
    if (!moved) continue;
    if (keep.empty()) {
      L.erase(L.begin() + (long)(i + 1));
    } else if (nx.kind == K_MULTI) {
      if (keep.size() == 1) {
        nx = std::move(keep[0]);
      } else {
        nx.parts = std::move(keep);
      }
    }
  }
}

void fuse_gemv_tails(Plan& p) {
  // opt-in (CLJXLA_B200_GEMV_TAIL=1): on Gemma-3-4B decode the two single-row
  // norms per layer as tails took 2.55 ms / step against 2.50 ms as their own
  // kernels, and the head norms, RoPE and GeGLU as tails 4.57 ms: the tail
  // waits for every CTA of the GEMV just as the kernel boundary does, and one
  // CTA runs what several did
  const char* e = getenv("CLJXLA_B200_GEMV_TAIL");
  if (!e || e[0] != '1') return;
  std::vector<Launch> out;
  out.reserve(p.launches.size());
  const size_t n = p.launches.size();
  for (size_t i = 0; i < n;) {
    Launch& l = p.launches[i];
    GemvParams g;
    if (l.kind != K_GEMV || l.blob.size() != sizeof(GemvParams) || !l.epi.empty()) {
      out.push_back(std::move(l));
      ++i;
      continue;
    }
    memcpy(&g, l.blob.data(), sizeof g);
    // the small programs right after the GEMV (flattening merged launches),
    // at most 8, up to the next launch of any other kind
    std::vector<Launch> tail;
    size_t j = i + 1;
    if (jit_gemv_tail_ok(g)) {
      for (; j < n; ++j) {
        Launch& t = p.launches[j];
        std::vector<Launch*> progs;
        if (t.kind == K_MULTI) {
          for (Launch& q : t.parts) progs.push_back(&q);
        } else {
          progs.push_back(&t);
        }
        bool ok = !progs.empty() && tail.size() + progs.size() <= 8;
        for (Launch* q : progs) ok = ok && jit_tail_program_ok(*q);
        if (!ok) break;
        for (Launch* q : progs) tail.push_back(std::move(*q));
      }
    }
    if (tail.empty()) {
      out.push_back(std::move(l));
      ++i;
      continue;
    }
    // the arrival counter: a zero word in the constant blob
    size_t off = (p.const_blob.size() + 255) & ~size_t(255);
    p.const_blob.resize(off + 4, 0);
    g.tail_ctr = DPtr{p.const_slot(), 0, (int64_t)off};
    Launch f;
    f.kind = K_GEMV_TAIL;
    f.blob.resize(sizeof g);
    memcpy(f.blob.data(), &g, sizeof g);
    f.label = l.label;
    f.algo_bytes = l.algo_bytes;
    f.algo_flops = l.algo_flops;
    for (Launch& t : tail) {
      f.label += "|" + t.label;
      f.algo_bytes += t.algo_bytes;
      f.algo_flops += t.algo_flops;
    }
    f.parts = std::move(tail);
    out.push_back(std::move(f));
    i = j;
  }
  p.launches = std::move(out);
}

void schedule_and_merge(Plan& p) {
  if (getenv("CLJXLA_B200_FOLD_KV") == nullptr || getenv("CLJXLA_B200_FOLD_KV")[0] != '0') fuse_dus_into_producers(p);
  // CLJXLA_B200_GEMV_PROLOGUE: 3 (default) the single-row norm producers only,
  // 1 every producer, 2 elementwise producers only, 0 none.  Measured on
  // Gemma-3-4B decode B=1: row producers as prologues 2.43 ms / step against
  // 2.50 ms as their own kernels; the GeGLU (elementwise) producers recomputed
  // in every CTA of the down projection cost more than they save (4.14 ms /
  // step for all producers against 3.37 ms with an earlier GEMV)
  {
    const char* e = getenv("CLJXLA_B200_GEMV_PROLOGUE");
    const char m = e && e[0] ? e[0] : '3';
    if (m == '1' || m == '2' || m == '3') fuse_gemv_prologues(p, m == '2', m == '3');
  }
  const int n = (int)p.launches.size();
  if (n < 2) return;
  std::vector<std::vector<Access>> acc(n);
  std::vector<char> known(n);
  for (int i = 0; i < n; ++i) known[i] = accesses(p, p.launches[i], acc[i]);
  // level = 1 + the deepest earlier launch it conflicts with (unknown kinds: barriers)
  std::vector<int> level(n, 0);
  int barrier = -1;  // index of the last unknown-kind launch
  for (int i = 0; i < n; ++i) {
    int lv = barrier >= 0 ? level[barrier] + 1 : 0;
    for (int j = std::max(0, barrier); j < i; ++j)
      if (!known[i] || !known[j] || conflict(acc[i], acc[j])) lv = std::max(lv, level[j] + 1);
    level[i] = lv;
    if (!known[i]) barrier = i;
  }
  std::vector<int> order(n);
  for (int i = 0; i < n; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return level[a] < level[b]; });
  if (const char* path = getenv("CLJXLA_B200_DUMP_SCHEDULE")) {
    if (FILE* f = fopen(path, "a")) {
      for (int i : order) {
        int kind = -1, block = 0, cluster = 0;
        merge_key(p.launches[i], &kind, &block, &cluster);
        fprintf(f, "%d\t%s\t%d\t%d\t%s\n", level[i], kernel_kind_name(p.launches[i].kind), block, cluster,
                p.launches[i].label.c_str());
      }
      fclose(f);
    }
  }
  std::vector<Launch> out;
  out.reserve(n);
  for (size_t k = 0; k < order.size();) {
    int kind, block, cluster;
    Launch& first = p.launches[order[k]];
    if (!merge_key(first, &kind, &block, &cluster)) {
      out.push_back(std::move(first));
      ++k;
      continue;
    }
    size_t e = k + 1;
    while (e < order.size() && e - k < JIT_MAXPARTS && level[order[e]] == level[order[k]]) {
      int k2, b2, c2;
      // row programs of one cluster shape merge at the largest block among them
      if (!merge_key(p.launches[order[e]], &k2, &b2, &c2) || k2 != kind || c2 != cluster ||
          (kind == K_EW && b2 != block))
        break;
      ++e;
    }
    if (e - k == 1) {
      out.push_back(std::move(first));
      ++k;
      continue;
    }
    Launch m;
    m.kind = K_MULTI;
    for (size_t q = k; q < e; ++q) {
      Launch& part = p.launches[order[q]];
      m.label += (m.label.empty() ? "" : "+") + part.label;
      m.algo_bytes += part.algo_bytes;
      m.algo_flops += part.algo_flops;
      m.parts.push_back(std::move(part));
    }
    out.push_back(std::move(m));
    k = e;
  }
  p.launches = std::move(out);
}

}  // namespace cljxla
