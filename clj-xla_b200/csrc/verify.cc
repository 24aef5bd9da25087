// Static bounds verification of a launch plan.  Every buffer a kernel can
// touch is described by a DPtr plus a strided extent; this checks, on the
// host and before anything runs, that each access region lies inside the
// buffer its argument-table slot will point at.  A planner bug therefore
// surfaces as an INTERNAL compile error rather than an out-of-bounds access
// on the device.
#include "fast_kernels.h"

namespace cljxla {
namespace {

size_t esz(int dt) { return dt_size((DT)dt); }

struct Checker {
  const Plan& p;
  const Launch* cur = nullptr;
  int64_t slot_bytes(int slot) const {
    int P = (int)p.params.size(), O = (int)p.outs.size();
    if (slot < 0) return -1;
    if (slot < P) return p.params[slot].bytes();
    if (slot < P + O) return p.outs[slot - P].bytes();
    int U = (int)p.inplace.size();
    if (slot < P + O + U) return p.inplace[slot - P - O].undo_bytes;
    if (slot == P + O + U) return (int64_t)p.const_blob.size();
    int b = slot - (P + O + U + 1);
    if (b < (int)p.tmp_bytes.size()) return p.tmp_bytes[b];
    if (slot == p.tmap_slot() && p.has_table()) return p.tmap_table_bytes();
    return -1;
  }
  void region(const DPtr& d, int64_t bytes, const char* what) const {
    if (bytes <= 0) return;
    int64_t cap = slot_bytes(d.slot);
    if (cap < 0 || d.off < 0 || d.off + bytes > cap)
      fail(E_INTERNAL, std::string("plan bounds check failed: ") + kernel_kind_name(cur->kind) + " '" +
                           cur->label + "' " + what + " slot " + std::to_string(d.slot) + " range [" +
                           std::to_string(d.off) + ", " + std::to_string(d.off + bytes) + ") exceeds buffer of " +
                           std::to_string(cap) + " bytes");
  }
  void view(const TView& v, const char* what) const {
    int64_t hi = 0;
    for (int i = 0; i < v.rank; ++i) {
      if (v.shape[i] == 0) return;
      if (v.stride[i] < 0) fail(E_INTERNAL, "negative stride in plan");
      hi += (v.shape[i] - 1) * v.stride[i];
    }
    region(v.p, (hi + 1) * (int64_t)esz(v.dt), what);
  }
  void strided(const DPtr& d, int dt, std::initializer_list<std::pair<int64_t, int64_t>> dims, const char* what) const {
    int64_t hi = 0;
    for (auto& ds : dims) {
      if (ds.first == 0) return;
      if (ds.second < 0) fail(E_INTERNAL, "negative stride in plan");
      hi += (ds.first - 1) * ds.second;
    }
    region(d, (hi + 1) * (int64_t)esz(dt), what);
  }
};

}  // namespace

namespace {
void verify_launch(const Plan& p, Checker& c, const Launch& l);
}

void verify_plan(const Plan& p) {
  Checker c{p};
  for (const Launch& l : p.launches) verify_launch(p, c, l);
}

namespace {
void verify_launch(const Plan& p, Checker& c, const Launch& l) {
  {
    if (l.kind == K_MULTI) {
      if (l.parts.size() < 2 || l.parts.size() > (size_t)JIT_MAXPARTS) fail(E_INTERNAL, "bad merged launch");
      for (const Launch& part : l.parts) verify_launch(p, c, part);
      return;
    }
    if (l.kind == K_FUSED_DUS) {
      if (l.parts.size() < 2 || (l.parts[0].kind != K_EW && l.parts[0].kind != K_ROWNORM) ||
          l.blob.size() != 4 * (l.parts.size() - 1))
        fail(E_INTERNAL, "bad folded KV write");
      for (const Launch& part : l.parts) {
        if (&part != &l.parts[0] && part.kind != K_DUS) fail(E_INTERNAL, "bad folded KV write");
        verify_launch(p, c, part);
      }
      return;
    }
    if (l.kind == K_GEMV_TAIL) {
      const GemvParams& g = *(const GemvParams*)l.blob.data();
      if (l.parts.empty()) fail(E_INTERNAL, "GEMV tail without programs");
      for (const Launch& part : l.parts) {
        if (part.kind != K_EW && part.kind != K_ROWNORM && part.kind != K_FUSED_DUS)
          fail(E_INTERNAL, "bad GEMV tail program");
        verify_launch(p, c, part);
      }
      c.cur = &l;
      c.region(g.tail_ctr, 4, "tail arrival counter");
    }
    if (!l.gtail.empty()) {  // row programs run by the CTAs completing their groups of GEMV rows
      if (l.kind != K_GEMV && l.kind != K_GEMV_FUSED) fail(E_INTERNAL, "group tails on a launch that is no GEMV");
      const GemvParams& g = *(const GemvParams*)l.blob.data();
      int64_t groups = 0;
      for (const Launch& q : l.gtail) {
        const Launch& qb = q.kind == K_FUSED_DUS ? q.parts[0] : q;
        if (qb.kind != K_ROWNORM || g.M != 1) fail(E_INTERNAL, "bad GEMV group tail");
        groups += ((const RowParams*)qb.blob.data())->rows;
        verify_launch(p, c, q);
      }
      c.cur = &l;
      c.region(g.tail_ctr, 4 * groups, "group-tail arrival counters");
    }
    if (!l.epi.empty() && l.kind == K_ROWNORM) {  // row program with an elementwise epilogue over its rows
      const Launch& e = l.epi[0];
      const Launch& eb = e.kind == K_FUSED_DUS ? e.parts[0] : e;
      if (l.epi.size() != 1 || eb.kind != K_EW ||
          ((const EwParams*)eb.blob.data())->n != ((const RowParams*)l.blob.data())->rows * ((const RowParams*)l.blob.data())->C)
        fail(E_INTERNAL, "bad row epilogue");
      verify_launch(p, c, e);
      c.cur = &l;
    } else if (!l.epi.empty()) {
      const GemvParams& g = *(const GemvParams*)l.blob.data();
      if ((l.kind != K_GEMV && l.kind != K_GEMV_FUSED) || l.epi.size() != 1 || l.epi[0].kind != K_EW || g.M != 1 ||
          g.nseg > 2 || (g.nseg == 2 && g.seg_end[1] != 2 * g.seg_end[0]) ||
          ((const EwParams*)l.epi[0].blob.data())->n != (g.nseg == 2 ? g.seg_end[0] : g.N))
        fail(E_INTERNAL, "bad GEMV epilogue");
      verify_launch(p, c, l.epi[0]);
      c.cur = &l;
    }
    if (l.kind == K_GEMV_FUSED) {
      if (l.parts.size() != 1 || (l.parts[0].kind != K_EW && l.parts[0].kind != K_ROWNORM))
        fail(E_INTERNAL, "bad GEMV prologue");
      const GemvParams& g = *(const GemvParams*)l.blob.data();
      if ((g.M > 1 && g.x_sm != g.K) || g.M * g.K * (int64_t)esz(g.x_dt) > 144 * 1024)
        fail(E_INTERNAL, "GEMV prologue x not dense or too large");
      verify_launch(p, c, l.parts[0]);
    }
    c.cur = &l;
    const void* b = l.blob.data();
    switch (l.kind) {
      case K_EW: {
        const EwParams& e = *(const EwParams*)b;
        if (e.n == 0) break;
        for (int i = 0; i < e.nin; ++i) {
          TView v{};
          v.p = e.in[i].p;
          v.dt = e.in[i].dt;
          v.rank = e.rank;
          for (int d = 0; d < e.rank; ++d) { v.shape[d] = e.dims[d]; v.stride[d] = e.in[i].stride[d]; }
          if (e.in[i].sel_dim >= 0) {  // concatenate operand: only its own index range is loaded
            const EwIn& in = e.in[i];
            if (in.sel_dim >= e.rank || in.sel_lo < 0 || in.sel_hi > e.dims[in.sel_dim] || in.sel_lo > in.sel_hi)
              fail(E_INTERNAL, "bad concatenate operand range");
            v.shape[in.sel_dim] = in.sel_hi - in.sel_lo;
          }
          c.view(v, "input");
        }
        for (int o = 0; o < e.nout; ++o) c.region(e.out[o].p, e.n * (int64_t)esz(e.out[o].dt), "output");
        for (int k = 0; k < e.ncode; ++k) {
          const EwInstr& I = e.code[k];
          if (I.dst >= EW_NREG || I.a >= EW_NREG || I.b >= EW_NREG || I.c >= EW_NREG)
            fail(E_INTERNAL, "register index out of range");
          if (I.op == EW_LOAD && I.aux >= e.nin) fail(E_INTERNAL, "load of a missing input");
          if (I.op == EW_IOTA && I.aux >= e.rank) fail(E_INTERNAL, "iota dimension out of range");
        }
        break;
      }
      case K_REDUCE: {
        const ReduceParams& r = *(const ReduceParams*)b;
        c.view(r.in, "input");
        c.region(r.out, r.n_out * (int64_t)esz(r.out_dt), "output");
        break;
      }
      case K_COPY: {
        const CopyParams& r = *(const CopyParams*)b;
        c.view(r.src, "source");
        c.view(r.dst, "destination");
        break;
      }
      case K_GATHER: {
        const GatherParams& g = *(const GatherParams*)b;
        c.strided(g.table, g.table_dt, {{g.rows_table, g.table_row_stride}, {g.row_len, 1}}, "table");
        c.view(g.idx, "indices");
        c.region(g.out, g.n_rows * g.row_len * (int64_t)esz(g.table_dt), "output");
        break;
      }
      case K_DUS: {
        const DusParams& d = *(const DusParams*)b;
        c.view(d.operand, "operand");
        c.view(d.update, "update");
        c.region(d.out, d.n * (int64_t)esz(d.dt), "output");
        if (d.has_undo) {
          int64_t nu = 1;
          for (int i = 0; i < d.rank; ++i) nu *= d.upd_shape[i];
          c.region(d.undo, 8 * CLJXLA_MAXR + nu * (int64_t)esz(d.dt), "undo record");
        }
        for (int i = 0; i < d.rank; ++i) {
          if (d.upd_shape[i] > d.out_shape[i]) fail(E_INVALID, "dynamic_update_slice update larger than operand");
          if (d.start_is_ptr[i]) c.region(d.start_ptr[i], (int64_t)esz(d.start_dt[i]), "start index");
        }
        break;
      }
      case K_ROWNORM: {
        const RowParams& r = *(const RowParams*)b;
        if (r.rows == 0) break;
        for (int i = 0; i < r.nin; ++i) {
          TView v{};
          v.p = r.in[i].p;
          v.dt = r.in[i].dt;
          v.rank = r.rank;
          for (int d = 0; d < r.rank; ++d) { v.shape[d] = r.dims[d]; v.stride[d] = r.in[i].stride[d]; }
          c.view(v, "input");
        }
        for (int o = 0; o < r.nout; ++o)
          c.region(r.out[o].p, (r.out[o].scalar ? r.rows : r.rows * r.C) * (int64_t)esz(r.out[o].dt), "output");
        if (r.nphase < 1 || r.nphase > RP_MAXPH) fail(E_INTERNAL, "bad row phase count");
        for (int ph = 0; ph < r.nphase; ++ph) {
          const RowPhase& P = r.ph[ph];
          if (P.lo > P.hi || P.hi > RP_MAXCODE || P.slo > P.shi || P.shi > RP_MAXCODE || P.red_reg >= RP_NREG ||
              P.red_dst >= RP_NREG)
            fail(E_INTERNAL, "bad row phase");
        }
        for (int k = 0; k < RP_MAXCODE; ++k) {
          const EwInstr& I = r.code[k];
          if (I.dst >= RP_NREG || I.a >= RP_NREG || I.b >= RP_NREG || I.c >= RP_NREG) fail(E_INTERNAL, "row register out of range");
          if (I.op == EW_LOAD && I.aux >= r.nin) fail(E_INTERNAL, "row load of a missing input");
        }
        break;
      }
      case K_GEMM: {
        const GemmParams& g = *(const GemmParams*)b;
        c.strided(g.a, g.a_dt, {{g.batch, g.a_sb}, {g.M, g.a_sm}, {g.K, g.a_sk}}, "lhs");
        c.strided(g.b, g.b_dt, {{g.batch, g.b_sb}, {g.K, g.b_sk}, {g.N, g.b_sn}}, "rhs");
        c.region(g.c, g.batch * g.M * g.N * (int64_t)esz(g.c_dt), "result");
        break;
      }
      case K_ALLREDUCE: {
        const AllReduceParams& a = *(const AllReduceParams*)b;
        if (a.ranks < 1 || a.count < 0) fail(E_INTERNAL, "bad all_reduce");
        c.region(a.src, a.count * (int64_t)esz(a.dt), "all_reduce source");
        c.region(a.dst, a.count * (int64_t)esz(a.dt), "all_reduce destination");
        break;
      }
      default:
        verify_fast_launch_impl(p, l, [&](const DPtr& d, int64_t bytes, const char* what) { c.region(d, bytes, what); });
        break;
    }
  }
}
}  // namespace

}  // namespace cljxla
