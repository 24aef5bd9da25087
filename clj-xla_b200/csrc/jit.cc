// Code generation and NVRTC compilation of fused kernels (see jit.h).
//
// The generated code is a transliteration of the interpreting kernels
// (ew_exec.cuh, k_generic.cu ew_kernel, k_row.cu row_kernel): the same
// per-op arithmetic, the same rounding to each op's printed element type,
// the same index decomposition and the same reduction order, with the
// program, shapes, strides and types fixed at compile time.
#include "jit.h"
#include "fast_kernels.h"
#include "sha256.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <sstream>
#include <thread>

namespace cljxla {
namespace {

// ------------------------------------------------------------------ prelude
const char* kPrelude = R"PRELUDE(
typedef unsigned int u32;
typedef long long i64;
typedef unsigned long long u64;
__device__ __forceinline__ unsigned short f2bf(float x) { unsigned short r; asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x)); return r; }
__device__ __forceinline__ unsigned short f2h(float x) { unsigned short r; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r) : "f"(x)); return r; }
__device__ __forceinline__ float h2f(unsigned short h) { float r; asm("cvt.f32.f16 %0, %1;" : "=f"(r) : "h"(h)); return r; }
__device__ __forceinline__ float rbf(float x) { return __uint_as_float((u32)f2bf(x) << 16); }
__device__ __forceinline__ float rh(float x) { return h2f(f2h(x)); }
__device__ __forceinline__ float F(u32 v) { return __uint_as_float(v); }
__device__ __forceinline__ u32 U(float v) { return __float_as_uint(v); }
__device__ __forceinline__ float fmax_nan(float x, float y) { return (x != x || y != y) ? __int_as_float(0x7fc00000) : fmaxf(x, y); }
__device__ __forceinline__ float fmin_nan(float x, float y) { return (x != x || y != y) ? __int_as_float(0x7fc00000) : fminf(x, y); }
// float -> i32 with truncation toward zero and saturation (NaN -> 0)
__device__ __forceinline__ int f2i_sat(float f) {
  if (f != f) return 0;
  if (f >= 2147483647.0f) return 2147483647;
  if (f <= -2147483648.0f) return (int)0x80000000;
  return (int)f;
}
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ u32 cluster_rank() { u32 r; asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r)); return r; }
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(const float* p, u32 rank) {
  u32 a = (u32)__cvta_generic_to_shared(p), b; float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(b) : "r"(a), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(b) : "memory");
  return v;
}
)PRELUDE";

bool is_float(int dt) { return dt == KDT_F32 || dt == KDT_BF16 || dt == KDT_F16 || dt == KDT_F64; }

std::string round_expr(const std::string& f, int dt) {
  if (dt == KDT_BF16) return "rbf(" + f + ")";
  if (dt == KDT_F16) return "rh(" + f + ")";
  return f;
}
std::string fbits(const std::string& f, int dt) { return "U(" + round_expr(f, dt) + ")"; }

std::string hex32(uint32_t v) {
  char b[16];
  snprintf(b, sizeof b, "0x%08xu", v);
  return b;
}

// buffer k of the launch: argument-table slot a.s[k] plus byte offset a.o[k]
// (a negative slot: a.o[k] is the address), so that programs that differ only
// in which buffers they touch compile to one kernel
std::string base_expr(int k) {
  std::ostringstream s;
  s << "((char*)(a.s[" << k << "] >= 0 ? argtab[a.s[" << k << "]] + (u64)a.o[" << k << "] : (u64)a.o[" << k << "]))";
  return s.str();
}

std::string args_struct() {
  return "struct JitArgs { int s[" + std::to_string(JIT_MAXBUF) + "]; int pad; long long o[" +
         std::to_string(JIT_MAXBUF) + "]; };\n";
}

// set while emitting the tail programs of a GEMV: their inputs include rows
// other CTAs of the same kernel wrote, so loads go through L2 (ld.global.cg)
thread_local bool g_l2_loads = false;

std::string load_expr(const std::string& base, const std::string& off, int dt) {
  if (g_l2_loads) {
    auto L = [&](const char* type) {
      return std::string("__ldcg((const ") + type + "*)(" + base + ") + (" + off + "))";
    };
    switch (dt) {
      case KDT_F32: return "U(" + L("float") + ")";
      case KDT_BF16: return "((u32)" + L("unsigned short") + " << 16)";
      case KDT_F16: return "U(h2f(" + L("unsigned short") + "))";
      case KDT_I32: case KDT_U32: return "(u32)" + L("int");
      case KDT_I8: return "(u32)(int)" + L("signed char");
      case KDT_U8: return "(u32)" + L("unsigned char");
      case KDT_I16: return "(u32)(int)" + L("short");
      case KDT_I1: return "(" + L("unsigned char") + " ? 1u : 0u)";
      case KDT_I64: return "(u32)(int)" + L("long long");
      case KDT_F64: return "U((float)" + L("double") + ")";
    }
  }
  const std::string o = "[" + off + "]";
  switch (dt) {
    case KDT_F32: return "U(((const float*)" + base + ")" + o + ")";
    case KDT_BF16: return "((u32)((const unsigned short*)" + base + ")" + o + " << 16)";
    case KDT_F16: return "U(h2f(((const unsigned short*)" + base + ")" + o + "))";
    case KDT_I32: case KDT_U32: return "(u32)((const int*)" + base + ")" + o;
    case KDT_I8: return "(u32)(int)((const signed char*)" + base + ")" + o;
    case KDT_U8: return "(u32)((const unsigned char*)" + base + ")" + o;
    case KDT_I16: return "(u32)(int)((const short*)" + base + ")" + o;
    case KDT_I1: return "(((const unsigned char*)" + base + ")" + o + " ? 1u : 0u)";
    case KDT_I64: return "(u32)(int)((const long long*)" + base + ")" + o;
    case KDT_F64: return "U((float)((const double*)" + base + ")" + o + ")";
  }
  fail(E_INTERNAL, "jit: load of an unknown element type");
}

std::string store_stmt(const std::string& base, const std::string& off, int dt, const std::string& v) {
  const std::string o = "[" + off + "]";
  switch (dt) {
    case KDT_F32: return "((float*)" + base + ")" + o + " = F(" + v + ");";
    case KDT_BF16: return "((unsigned short*)" + base + ")" + o + " = f2bf(F(" + v + "));";
    case KDT_F16: return "((unsigned short*)" + base + ")" + o + " = f2h(F(" + v + "));";
    case KDT_I32: case KDT_U32: return "((int*)" + base + ")" + o + " = (int)" + v + ";";
    case KDT_I8: return "((signed char*)" + base + ")" + o + " = (signed char)(int)" + v + ";";
    case KDT_U8: return "((unsigned char*)" + base + ")" + o + " = (unsigned char)" + v + ";";
    case KDT_I16: return "((short*)" + base + ")" + o + " = (short)(int)" + v + ";";
    case KDT_I1: return "((unsigned char*)" + base + ")" + o + " = " + v + " ? 1 : 0;";
    case KDT_I64: return "((long long*)" + base + ")" + o + " = (long long)(int)" + v + ";";
    case KDT_F64: return "((double*)" + base + ")" + o + " = (double)F(" + v + ");";
  }
  fail(E_INTERNAL, "jit: store of an unknown element type");
}

std::string convert_expr(const std::string& v, int from, int to) {
  const bool ff = is_float(from), tf = is_float(to);
  if (to == KDT_I1) return ff ? "(F(" + v + ") != 0.0f ? 1u : 0u)" : "(" + v + " != 0u ? 1u : 0u)";
  if (ff && tf) return fbits("F(" + v + ")", to);
  if (!ff && tf) return fbits(from == KDT_U32 ? "(float)" + v : "(float)(int)" + v, to);
  std::string r = ff ? "f2i_sat(F(" + v + "))" : "(int)" + v;
  if (to == KDT_I8) r = "(int)(signed char)" + r;
  else if (to == KDT_U8) r = "(int)(unsigned char)" + r;
  else if (to == KDT_I16) r = "(int)(short)" + r;
  return "(u32)(" + r + ")";
}

// Emits one program step as "u32 <name> = ...;".  reg[] maps register -> the
// expression currently holding it; x[] names the loop index per dimension.
struct Emitter {
  std::ostringstream& s;
  const EwIn* ins;
  int rank;
  std::vector<std::string> x;  // index variable per loop dim
  std::vector<std::string> in_base;
  int counter = 0;
  // per-thread register cache of loaded inputs (row bodies whose row fits a few
  // elements per thread): input i element jj lives in cache_arr[i][cache_j]
  std::vector<std::string> cache_arr;
  std::string cache_j;
  std::vector<char> cached;

  std::string reg_or_zero(const std::vector<std::string>& reg, int r) {
    return (r >= 0 && r < (int)reg.size() && !reg[r].empty()) ? reg[r] : std::string("0u");
  }

  std::string offset(const EwIn& in, int skip_dim, const std::string& extra) {
    std::ostringstream o;
    bool any = false;
    for (int d = 0; d < rank; ++d) {
      if (d == skip_dim || in.stride[d] == 0) continue;
      if (any) o << " + ";
      o << x[d] << " * " << in.stride[d] << "LL";
      any = true;
    }
    if (!extra.empty()) {
      if (any) o << " + ";
      o << extra;
      any = true;
    }
    if (!any) o << "0";
    return o.str();
  }

  void step(const EwInstr& I, std::vector<std::string>& reg, const std::string& indent) {
    const std::string v = "v" + std::to_string(counter++);
    const int dt = I.dt;
    const bool fl = is_float(dt);
    auto A = [&] { return reg_or_zero(reg, I.a); };
    auto B = [&] { return reg_or_zero(reg, I.b); };
    auto C = [&] { return reg_or_zero(reg, I.c); };
    std::string e;
    switch (I.op) {
      case EW_LOAD: {
        const EwIn& in = ins[I.aux];
        const std::string& base = in_base[I.aux];
        if (in.sel_dim >= 0) {
          const std::string& k = x[in.sel_dim];
          const std::string extra = "(" + k + " - " + std::to_string(in.sel_lo) + "LL) * " +
                                    std::to_string(in.stride[in.sel_dim]) + "LL";
          s << indent << "u32 " << v << ";\n"
            << indent << "if (" << k << " >= " << in.sel_lo << "LL && " << k << " < " << in.sel_hi << "LL) " << v
            << " = " << load_expr(base, offset(in, in.sel_dim, extra), in.dt) << ";\n"
            << indent << "else " << v << " = " << B() << ";\n";
          reg[I.dst] = v;
          return;
        }
        e = load_expr(base, offset(in, -1, ""), in.dt);
        if (I.aux < (int)cache_arr.size() && !cache_arr[I.aux].empty()) {
          const std::string slot = cache_arr[I.aux] + "[" + cache_j + "]";
          if (!cached[I.aux]) {  // first phase to read it loads it; later phases reuse the register
            s << indent << slot << " = " << e << ";\n";
            cached[I.aux] = 1;
          }
          e = slot;
        }
        break;
      }
      case EW_IMM: e = fl ? hex32(*(const uint32_t*)&I.fimm) : "(u32)" + std::to_string(I.iimm); break;
      case EW_IOTA: e = fl ? fbits("(float)" + x[I.aux], dt) : "(u32)" + x[I.aux]; break;
      case EW_ADD: case EW_SUB: case EW_MUL: case EW_DIV: case EW_MAX: case EW_MIN: {
        if (fl) {
          const std::string fa = "F(" + A() + ")", fb = "F(" + B() + ")";
          std::string z;
          switch (I.op) {
            case EW_ADD: z = "(" + fa + " + " + fb + ")"; break;
            case EW_SUB: z = "(" + fa + " - " + fb + ")"; break;
            case EW_MUL: z = "(" + fa + " * " + fb + ")"; break;
            case EW_DIV: z = "(" + fa + " / " + fb + ")"; break;
            case EW_MAX: z = "fmax_nan(" + fa + ", " + fb + ")"; break;
            default: z = "fmin_nan(" + fa + ", " + fb + ")"; break;
          }
          e = fbits(z, dt);
        } else {
          const std::string ia = "(int)" + A(), ib = "(int)" + B();
          std::string z;
          switch (I.op) {
            case EW_ADD: z = "(" + ia + " + " + ib + ")"; break;
            case EW_SUB: z = "(" + ia + " - " + ib + ")"; break;
            case EW_MUL: z = "(" + ia + " * " + ib + ")"; break;
            case EW_DIV: z = "(" + ib + " == 0 ? -1 : " + ia + " / " + ib + ")"; break;
            case EW_MAX: z = "max(" + ia + ", " + ib + ")"; break;
            default: z = "min(" + ia + ", " + ib + ")"; break;
          }
          if (dt == KDT_I1) z = "(" + z + " ? 1 : 0)";
          e = "(u32)" + z;
        }
        break;
      }
      case EW_EXP: case EW_TANH: case EW_SQRT: case EW_RSQRT: case EW_SIN: case EW_COS:
      case EW_LOGISTIC: case EW_NEG: case EW_ABS: {
        if (fl) {
          const std::string fx = "F(" + A() + ")";
          std::string z;
          switch (I.op) {
            case EW_EXP: z = "expf(" + fx + ")"; break;
            case EW_TANH: z = "tanhf(" + fx + ")"; break;
            case EW_SQRT: z = "sqrtf(" + fx + ")"; break;
            case EW_RSQRT: z = "(1.0f / sqrtf(" + fx + "))"; break;
            case EW_SIN: z = "sinf(" + fx + ")"; break;
            case EW_COS: z = "cosf(" + fx + ")"; break;
            case EW_LOGISTIC: z = "(1.0f / (1.0f + expf(-" + fx + ")))"; break;
            case EW_NEG: z = "(-" + fx + ")"; break;
            default: z = "fabsf(" + fx + ")"; break;
          }
          e = fbits(z, dt);
        } else {
          const std::string ix = "(int)" + A();
          if (I.op == EW_NEG) e = "(u32)(-" + ix + ")";
          else if (I.op == EW_ABS) e = "(u32)(" + ix + " < 0 ? -" + ix + " : " + ix + ")";
          else e = "(u32)" + ix;
        }
        break;
      }
      case EW_CONVERT: e = convert_expr(A(), I.aux, dt); break;
      case EW_CMP: {
        static const char* ops[] = {"==", "!=", ">=", ">", "<=", "<"};
        const char* op = ops[I.aux < 6 ? I.aux : 5];
        if (is_float(I.aux2)) e = "((F(" + A() + ") " + op + " F(" + B() + ")) ? 1u : 0u)";
        else e = "(((int)" + A() + " " + op + " (int)" + B() + ") ? 1u : 0u)";
        break;
      }
      case EW_SELECT: e = "(" + A() + " ? " + B() + " : " + C() + ")"; break;
      default: fail(E_INTERNAL, "jit: unknown program step");
    }
    s << indent << "const u32 " << v << " = " << e << ";\n";
    reg[I.dst] = v;
  }
};

}  // namespace

// Options of an emitted program body: the CTA size its loops stride by, and
// (smem_out >= 0) an output that is also written to shared memory at xsb,
// with the global stores only where gst holds (a GEMV prologue, in which every
// CTA runs the whole program and one CTA stores its results).
// A KV-window write folded into the program producing its update: output
// `out` (element e of the dense update) also goes to the in-place cache at the
// clamped start indices, after the window's old value is saved to the undo
// record (same thread, so old-before-new holds per element).
struct DusStore {
  int out = -1;
  DusParams d{};
  int b_cache = -1, b_undo = -1;
  int b_start[CLJXLA_MAXR] = {};
};

struct BodyOpts {
  int block = 256;
  int row_cache = 4;  // row programs keep their inputs in registers for rows of up to row_cache * block elements
  int smem_out = -1;
  std::string sync = "__syncthreads()";  // barrier over the threads running the body
  std::vector<DusStore> dus;
  // elementwise body over the element range [e0, e1) given as arguments (a GEMV
  // epilogue) instead of a grid-stride share of every element
  bool ranged = false;
};

// clamped start indices of each folded KV write (and, CTA 0, its undo header)
void emit_dus_prelude(std::ostringstream& s, const BodyOpts& bo, const std::string& ind) {
  for (size_t k = 0; k < bo.dus.size(); ++k) {
    const DusStore& u = bo.dus[k];
    for (int d = 0; d < u.d.rank; ++d) {
      const std::string v = "dst" + std::to_string(k) + "_" + std::to_string(d);
      const int64_t hi = u.d.out_shape[d] - u.d.upd_shape[d];
      if (u.d.start_is_ptr[d])
        s << ind << "i64 " << v << " = (i64)(int)" << load_expr(base_expr(u.b_start[d]), "0", u.d.start_dt[d]) << ";\n";
      else
        s << ind << "i64 " << v << " = " << u.d.start_imm[d] << "LL;\n";
      s << ind << v << " = " << v << " < 0 ? 0 : (" << v << " > " << hi << "LL ? " << hi << "LL : " << v << ");\n";
    }
    if (u.b_undo >= 0) {
      s << ind << "if (bid == 0u && threadIdx.x == 0) {\n";
      for (int d = 0; d < CLJXLA_MAXR; ++d)
        s << ind << "  ((long long*)" << base_expr(u.b_undo) << ")[" << d << "] = "
          << (d < u.d.rank ? "dst" + std::to_string(k) + "_" + std::to_string(d) : std::string("0")) << ";\n";
      s << ind << "}\n";
    }
  }
}

// the folded KV writes of output o for update element e holding value v
void emit_dus_stores(std::ostringstream& s, const BodyOpts& bo, int o, const std::string& e, const std::string& v,
                     const std::string& ind) {
  for (size_t k = 0; k < bo.dus.size(); ++k) {
    const DusStore& u = bo.dus[k];
    if (u.out != o) continue;
    s << ind << "{\n" << ind << "  i64 rem = " << e << ", off = 0;\n";
    int64_t ostride = 1;
    for (int d = u.d.rank - 1; d >= 0; --d) {
      s << ind << "  { const i64 i = rem % " << u.d.upd_shape[d] << "LL; rem /= " << u.d.upd_shape[d] << "LL; off += (dst" << k
        << "_" << d << " + i) * " << ostride << "LL; }\n";
      ostride *= u.d.out_shape[d];
    }
    const std::string cache = base_expr(u.b_cache);
    if (u.b_undo >= 0)
      s << ind << "  " << store_stmt("(" + base_expr(u.b_undo) + " + " + std::to_string(8 * CLJXLA_MAXR) + ")", e, u.d.dt,
                                     load_expr(cache, "off", u.d.dt))
        << "\n";
    // the update's own rounding first (the value the DUS would have read), then the cache type's
    const std::string vu = u.d.update.dt == u.d.dt ? v : fbits("F(" + v + ")", u.d.update.dt);
    s << ind << "  " << store_stmt(cache, "off", u.d.dt, vu) << "\n" << ind << "}\n";
  }
}

// ------------------------------------------------------------------ elementwise
// The program of one elementwise launch as a device function over blocks
// [0, nblk) (bid = this CTA's block in that range).
void emit_ew_body(std::ostringstream& s, const EwParams& P, const std::string& fname, const BodyOpts& bo) {
  s << "__device__ __forceinline__ void " << fname << "(const u64* __restrict__ argtab, const JitArgs& a, "
    << (bo.ranged ? "i64 e0, i64 e1" : "unsigned bid, unsigned nblk")
    << (bo.smem_out >= 0 ? ", char* __restrict__ xsb, bool gst" : "") << ") {\n";
  Emitter em{s, P.in, P.rank};
  for (int i = 0; i < P.nin; ++i) {
    em.in_base.push_back("in" + std::to_string(i));
    s << "  const char* in" << i << " = " << base_expr(i) << ";\n";
  }
  for (int o = 0; o < P.nout; ++o) s << "  char* out" << o << " = " << base_expr(P.nin + o) << ";\n";
  if (bo.ranged) s << "  const unsigned bid = e0 == 0 ? 0u : 1u;  // (the range holding element 0 writes undo headers)\n";
  emit_dus_prelude(s, bo, "  ");
  if (bo.ranged)
    s << "  for (i64 e = e0 + threadIdx.x; e < e1; e += " << bo.block << ") {\n";
  else
    s << "  for (i64 e = (i64)bid * " << bo.block << " + threadIdx.x; e < " << P.n << "LL; e += (i64)nblk * "
      << bo.block << ") {\n";
  for (int d = 0; d < P.rank; ++d) em.x.push_back("x" + std::to_string(d));
  if (P.rank == 1) {
    s << "    const i64 x0 = e;\n";
  } else {
    s << "    i64 rem = e;\n";
    for (int d = P.rank - 1; d > 0; --d)
      s << "    const i64 x" << d << " = rem % " << P.dims[d] << "LL; rem /= " << P.dims[d] << "LL;\n";
    s << "    const i64 x0 = rem;\n";
  }
  std::vector<std::string> reg(EW_NREG);
  for (int pc = 0; pc < P.ncode; ++pc) em.step(P.code[pc], reg, "    ");
  for (int o = 0; o < P.nout; ++o) {
    const std::string v = em.reg_or_zero(reg, P.out[o].reg);
    s << "    " << (bo.smem_out >= 0 ? "if (gst) " : "") << store_stmt("out" + std::to_string(o), "e", P.out[o].dt, v)
      << "\n";
    if (o == bo.smem_out) s << "    " << store_stmt("xsb", "e", P.out[o].dt, v) << "\n";
    emit_dus_stores(s, bo, o, "e", v, "    ");
  }
  s << "  }\n}\n";
}

std::string jit_source_ew(const EwParams& P) {
  std::ostringstream s;
  s << kPrelude << args_struct();
  emit_ew_body(s, P, "ew_body", BodyOpts{});
  s << "extern \"C\" __global__ void __launch_bounds__(256) cljxla_fused_ew(const u64* __restrict__ argtab, "
       "const JitArgs a) {\n  pdl_enter();\n  ew_body(argtab, a, blockIdx.x, gridDim.x);\n}\n";
  return s.str();
}

// ------------------------------------------------------------------ row regions
void row_launch_shape(const RowParams& p, int* block, int* cluster, int64_t* grid) {
  // A decode row (a few thousand elements) is latency-bound: one CTA of up to
  // 1024 threads reduces it fastest (a cluster adds a DSMEM barrier per phase,
  // measured at ~9.6 us per 2560-wide norm against a few us for one CTA).
  // Clusters only for very long rows, where one SM's bandwidth would limit.
  int cl = 1;
  if (p.C >= 8192)
    while (cl < 8 && p.rows * cl * 2 <= 2 * 148 && p.C / (cl * 2) >= 1024) cl *= 2;
  if (cl > 1) {
    const int64_t cols = (p.C + cl - 1) / cl;
    *block = cols <= 256 ? 256 : cols <= 512 ? 512 : 1024;
    *grid = p.rows * cl;
  } else {
    *block = p.C >= 2048 ? 1024 : p.C >= 1024 ? 512 : p.C >= 256 ? 128 : 64;
    *grid = p.rows < 65535 ? p.rows : 65535;
  }
  *cluster = cl;
}

void emit_row_body(std::ostringstream& s, const RowParams& P, int BLOCK, int CL, const std::string& fname,
                   const BodyOpts& bo) {
  s << "__device__ __forceinline__ void " << fname
    << "(const u64* __restrict__ argtab, const JitArgs& a, unsigned bid, unsigned nblk"
    << (bo.smem_out >= 0 ? ", char* __restrict__ xsb, bool gst" : "") << ") {\n";
  s << "  __shared__ float red_f[" << BLOCK / 32 << "];\n  __shared__ float bcast;\n  __shared__ float cl_part["
    << RP_MAXPH << "];\n";
  s << "  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;\n";
  s << "  const u32 crank = " << (CL > 1 ? "cluster_rank()" : "0u") << ";\n";
  const int64_t Cc = (P.C + CL - 1) / CL;
  s << "  const i64 c0 = (i64)crank * " << Cc << "LL;\n";
  s << "  const i64 c1 = min((i64)" << P.C << "LL, c0 + " << Cc << "LL);\n";
  Emitter em{s, P.in, P.rank};
  for (int i = 0; i < P.nin; ++i) {
    em.in_base.push_back("in" + std::to_string(i));
    s << "  const char* in" << i << " = " << base_expr(i) << ";\n";
  }
  for (int o = 0; o < P.nout; ++o) s << "  char* out" << o << " = " << base_expr(P.nin + o) << ";\n";
  s << "  (void)lane; (void)warp; (void)c1;\n";
  emit_dus_prelude(s, bo, "  ");
  s << "  for (i64 row = bid / " << CL << "; row < " << P.rows << "LL; row += nblk / " << CL << ") {\n";
  for (int d = 0; d < P.rank; ++d) em.x.push_back("x" + std::to_string(d));
  s << "    i64 rem = row;\n";
  for (int d = P.rank - 2; d >= 0; --d)
    s << "    const i64 x" << d << " = rem % " << P.dims[d] << "LL; rem /= " << P.dims[d] << "LL;\n";
  s << "    (void)rem;\n";
  // per-row scalars live for the whole row
  std::vector<std::string> sreg(RP_NREG);
  for (int r = RP_SREG0; r < RP_NREG; ++r) s << "    u32 s" << r << " = 0u; (void)s" << r << ";\n";
  for (int r = RP_SREG0; r < RP_NREG; ++r) sreg[r] = "s" + std::to_string(r);
  const std::string xc = "x" + std::to_string(P.rank - 1);
  // a row of a few elements per thread: every phase walks the same J elements,
  // so the inputs are loaded once (first phase) and kept in registers
  const int J = (CL == 1 && Cc <= (int64_t)bo.row_cache * BLOCK) ? (int)((Cc + BLOCK - 1) / BLOCK) : 0;
  if (J > 0) {
    em.cache_arr.assign(P.nin, std::string());
    em.cached.assign(P.nin, 0);
    em.cache_j = "jj";
    for (int i = 0; i < P.nin; ++i)
      if (P.in[i].sel_dim < 0) {
        em.cache_arr[i] = "cin" + std::to_string(i);
        s << "    u32 cin" << i << "[" << J << "];\n";
      }
  }
  for (int ph = 0; ph < P.nphase; ++ph) {
    const RowPhase& Ph = P.ph[ph];
    const bool sum = Ph.red_kind == 0;
    s << "    {  // phase " << ph << "\n";
    s << "      float acc = " << (sum ? "0.0f" : "-__int_as_float(0x7f800000)") << ";\n";
    if (J > 0)
      s << "#pragma unroll\n      for (int jj = 0; jj < " << J << "; ++jj) {\n        const i64 " << xc
        << " = c0 + threadIdx.x + (i64)jj * " << BLOCK << ";\n        if (" << xc << " < c1) {\n";
    else
      s << "      for (i64 " << xc << " = c0 + threadIdx.x; " << xc << " < c1; " << xc << " += " << BLOCK << ") {\n";
    std::vector<std::string> reg = sreg;  // per-element registers start undefined
    if (J > 0 && ph == 0)  // every cached input in flight at once, before any phase needs it
      for (int i = 0; i < P.nin; ++i)
        if (!em.cache_arr[i].empty() && !em.cached[i]) {
          s << "        " << em.cache_arr[i] << "[jj] = "
            << load_expr(em.in_base[i], em.offset(P.in[i], -1, ""), P.in[i].dt) << ";\n";
          em.cached[i] = 1;
        }
    for (int pc = Ph.lo; pc < Ph.hi; ++pc) em.step(P.code[pc], reg, "        ");
    if (Ph.red_reg >= 0) {
      const std::string xv = "F(" + em.reg_or_zero(reg, Ph.red_reg) + ")";
      s << "        acc = " << (sum ? "acc + " + xv : "fmaxf(acc, " + xv + ")") << ";\n";
    }
    for (int o = 0; o < P.nout; ++o)
      if (!P.out[o].scalar && P.out[o].phase == ph) {
        const std::string off = "row * " + std::to_string(P.C) + "LL + " + xc;
        const std::string v = em.reg_or_zero(reg, P.out[o].reg);
        s << "        " << (bo.smem_out >= 0 ? "if (gst) " : "")
          << store_stmt("out" + std::to_string(o), off, P.out[o].dt, v) << "\n";
        if (o == bo.smem_out) s << "        " << store_stmt("xsb", off, P.out[o].dt, v) << "\n";
        emit_dus_stores(s, bo, o, off, v, "        ");
      }
    s << (J > 0 ? "        }\n      }\n" : "      }\n");
    if (Ph.red_reg >= 0) {
      const std::string comb = sum ? "t = t + o;" : "t = fmaxf(t, o);";
      s << "      for (int sh = 16; sh > 0; sh >>= 1) { float o = __shfl_xor_sync(0xffffffffu, acc, sh); "
        << (sum ? "acc = acc + o;" : "acc = fmaxf(acc, o);") << " }\n";
      s << "      if (lane == 0) red_f[warp] = acc;\n      " << bo.sync << ";\n";
      s << "      float t = " << (sum ? "0.0f" : "-__int_as_float(0x7f800000)") << ";\n";
      s << "      if (threadIdx.x == 0) for (int w = 0; w < " << BLOCK / 32 << "; ++w) { float o = red_f[w]; " << comb
        << " }\n";
      if (CL > 1) {
        s << "      if (threadIdx.x == 0) cl_part[" << ph << "] = t;\n      cluster_sync();\n";
        s << "      if (threadIdx.x == 0) { t = " << (sum ? "0.0f" : "-__int_as_float(0x7f800000)") << "; for (u32 r = 0; r < "
          << CL << "; ++r) { float o = ld_cluster_f32(&cl_part[" << ph << "], r); " << comb << " } }\n";
      }
      s << "      if (threadIdx.x == 0) { float o = __uint_as_float(" << hex32(*(const uint32_t*)&Ph.red_init) << "); "
        << comb << " bcast = " << round_expr("t", Ph.red_dt) << "; }\n";
      s << "      " << bo.sync << ";\n      s" << (int)Ph.red_dst << " = U(bcast);\n      " << bo.sync << ";\n";
    }
    // per-row scalar program after this phase (its immediates use fresh names)
    std::vector<std::string> sc = sreg;
    for (int pc = Ph.slo; pc < Ph.shi; ++pc) {
      const EwInstr& I = P.code[pc];
      if (I.dst >= RP_SREG0) {
        // scalar results keep their fixed names
        std::vector<std::string> tmp = sc;
        em.step(I, tmp, "      ");
        s << "      s" << (int)I.dst << " = " << tmp[I.dst] << ";\n";
      } else {
        em.step(I, sc, "      ");
      }
    }
    s << "    }\n";
  }
  s << "    if (threadIdx.x == 0 && crank == 0u" << (bo.smem_out >= 0 ? " && gst" : "") << ") {\n";
  for (int o = 0; o < P.nout; ++o)
    if (P.out[o].scalar)
      s << "      " << store_stmt("out" + std::to_string(o), "row", P.out[o].dt, sreg[P.out[o].reg]) << "\n";
  s << "    }\n  }\n";
  if (CL > 1) s << "  cluster_sync();\n";
  s << "}\n";
}

std::string jit_source_row(const RowParams& P, int BLOCK, int CL) {
  std::ostringstream s;
  s << kPrelude << args_struct();
  emit_row_body(s, P, BLOCK, CL, "row_body", BodyOpts{});
  s << "extern \"C\" __global__ void __launch_bounds__(" << BLOCK
    << ") cljxla_fused_row(const u64* __restrict__ argtab, const JitArgs a) {\n  pdl_enter();\n"
       "  row_body(argtab, a, blockIdx.x, gridDim.x);\n}\n";
  return s.str();
}

namespace {

// shape and buffers of one elementwise / row launch; false for other kinds
int program_buffers(const Launch& l) {
  if (l.kind == K_EW) return ((const EwParams*)l.blob.data())->nin + ((const EwParams*)l.blob.data())->nout;
  if (l.kind == K_ROWNORM) return ((const RowParams*)l.blob.data())->nin + ((const RowParams*)l.blob.data())->nout;
  return -1;
}

// the folded KV writes of a K_FUSED_DUS launch, with their buffers numbered
// after the producer's; empty when they do not fit the argument block
std::vector<DusStore> dus_stores_of(const Launch& l) {
  std::vector<DusStore> out;
  int k = program_buffers(l.parts[0]);
  const int32_t* outs = (const int32_t*)l.blob.data();
  if (k < 0 || l.blob.size() != 4 * (l.parts.size() - 1)) return {};
  for (size_t i = 1; i < l.parts.size(); ++i) {
    DusStore u;
    u.out = outs[i - 1];
    memcpy(&u.d, l.parts[i].blob.data(), sizeof(DusParams));
    u.b_cache = k++;
    if (u.d.has_undo) u.b_undo = k++;
    for (int d = 0; d < u.d.rank; ++d)
      if (u.d.start_is_ptr[d]) u.b_start[d] = k++;
    out.push_back(u);
  }
  if (k > JIT_MAXBUF) return {};
  return out;
}

bool describe_one(const Launch& l, int64_t* grid, int* block, int* cluster, JitArgs* args) {
  *args = JitArgs{};
  auto put = [&](int k, const DPtr& p) {
    args->s[k] = p.slot;
    args->o[k] = p.off;
  };
  if (l.kind == K_EW) {
    const EwParams& e = *(const EwParams*)l.blob.data();
    if (e.n == 0 || e.nin + e.nout > JIT_MAXBUF) return false;
    int64_t g = (e.n + 255) / 256;
    *grid = g > 148 * 64 ? 148 * 64 : (g < 1 ? 1 : g);
    *block = 256;
    *cluster = 1;
    for (int i = 0; i < e.nin; ++i) put(i, e.in[i].p);
    for (int o = 0; o < e.nout; ++o) put(e.nin + o, e.out[o].p);
    return true;
  }
  if (l.kind == K_ROWNORM) {
    const RowParams& r = *(const RowParams*)l.blob.data();
    if (r.rows == 0 || r.nin + r.nout > JIT_MAXBUF) return false;
    row_launch_shape(r, block, cluster, grid);
    for (int i = 0; i < r.nin; ++i) put(i, r.in[i].p);
    for (int o = 0; o < r.nout; ++o) put(r.nin + o, r.out[o].p);
    return true;
  }
  if (l.kind == K_FUSED_DUS) {
    if (l.parts.size() < 2 || !describe_one(l.parts[0], grid, block, cluster, args)) return false;
    const std::vector<DusStore> ds = dus_stores_of(l);
    if (ds.empty()) return false;
    for (const DusStore& u : ds) {
      put(u.b_cache, u.d.out);
      if (u.b_undo >= 0) put(u.b_undo, u.d.undo);
      for (int d = 0; d < u.d.rank; ++d)
        if (u.d.start_is_ptr[d]) put(u.b_start[d], u.d.start_ptr[d]);
    }
    return true;
  }
  return false;
}

void emit_body(std::ostringstream& s, const Launch& l, int block, int cluster, const std::string& fname,
               const BodyOpts& bo = BodyOpts{});

// SM count of the current device; 148 (B200) when planning on a host without a GPU
int sm_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) {
    cudaGetLastError();
    return 148;
  }
  return device_sm_count();
}

// Decode GEMV fed by bulk copies (K_GEMV, and K_GEMV_FUSED with its producer
// as a prologue).  One CTA per SM owns a contiguous range of weight rows (the
// segments' rows laid end to end).  A producer warp streams the range through
// a ring of shared-memory stages with cp.async.bulk (each stage: RPS whole
// rows, completion counted on an mbarrier), starting before the dependency
// wait, since weights are never written by a plan kernel; 8 consumer warps
// compute one row part each per stage (WPR warps per row) from shared memory
// and release the stage.  x lives in shared memory, in x's element type: read
// from memory, or computed by the producer's program in every CTA (CTA 0 also
// stores the producer's outputs).  Every mbarrier wait is bounded; a timeout
// sets the plan's status word and the CTA stops, after the producer has
// waited (bounded) for its copies in flight.
struct GemvGeometry {
  int wpr, rps, nstage, stage_bytes, x_bytes, ctas_per_sm;
};

// CTAs per SM of the bulk-copy GEMV (CLJXLA_B200_GEMV_CTAS, 1 or 2): two halve
// each CTA's ring so that two pipelines share an SM
int gemv_ctas_per_sm() {
  static const int n = [] {
    const char* e = getenv("CLJXLA_B200_GEMV_CTAS");
    return e && e[0] == '2' ? 2 : 1;
  }();
  return n;
}

bool gemv_tma_geometry(const GemvParams& G, GemvGeometry* g) {
  constexpr int WARPS = 8;
  if (G.M < 1 || G.M > 8 || G.K % 8 != 0) return false;
  int wpr = 1;
  while (wpr < WARPS && (G.K / wpr > 2560 || (G.K / wpr) % 8 != 0)) wpr *= 2;
  if (G.K % wpr != 0 || (G.K / wpr) % 8 != 0 || G.K / wpr > 4096) return false;
  g->wpr = wpr;
  g->rps = WARPS / wpr;
  g->stage_bytes = (int)(g->rps * G.K * 2);
  g->x_bytes = (int)(G.M * G.K * (G.x_dt == KDT_F32 ? 4 : 2));
  if (g->x_bytes > 64 * 1024) return false;
  g->ctas_per_sm = gemv_ctas_per_sm();
  const int budget = (g->ctas_per_sm == 2 ? 108 : 200) * 1024 - g->x_bytes;
  g->nstage = std::min(4, budget / g->stage_bytes);
  return g->nstage >= 2;
}

// device helpers of the batched (tensor-core) GEMV kernels
std::string gemv_mma_helpers() {
  return std::string(R"G(__device__ __forceinline__ u32 sa(const void* p) { return (u32)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mb_init(u32 a, u32 n) { asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(n)); }
__device__ __forceinline__ void mb_expect(u32 a, u32 bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(u32 a) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory"); }
__device__ __forceinline__ bool mb_try(u32 a, u32 parity) {
  u32 ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(a), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mb_wait(u32 a, u32 parity) {
  for (u32 i = 0; i < (1u << 22); ++i)
    if (mb_try(a, parity)) return true;
  return false;
}
__device__ __forceinline__ void bulk_g2s(u32 dst, const void* src, u32 bytes, u32 bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ u32 lds32(u32 a) { u32 v; asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a)); return v; }
__device__ __forceinline__ void ldsm_x2(u32 a, u32& r0, u32& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(a));
}
__device__ __forceinline__ void mma16816(float* c, u32 a0, u32 a2, u32 b0, u32 b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3]) : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ bool consumers_any(bool p) {
  u32 r;
  asm volatile("{\n\t.reg .pred q, o;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred o, 1, 256, q;\n\tselp.u32 %0, 1, 0, o;\n\t}"
               : "=r"(r) : "r"((u32)p) : "memory");
  return r != 0;
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ float2 lds64f(u32 a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ u32 pack2(float lo, float hi) { u32 r; asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo)); return r; }
__device__ __forceinline__ float lo_bf(u32 v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hi_bf(u32 v) { return __uint_as_float(v & 0xffff0000u); }
)G");
}

// Batched decode rows (2 <= M <= 8) on the tensor cores: the same bulk-copy
// ring, 8 weight rows per stage (one 8-column mma tile; each row copied to a
// 16-byte-padded shared row so ldmatrix is conflict-free), x in shared memory
// as bf16 (f32 x as an exact hi + mid + lo split), the 8 consumer warps each
// covering an eighth of K with mma.sync m16n8k16 (rows M..15 of the A tile are
// zero) and summing their partials through shared memory per stage.
bool describe_gemv_mma(const GemvParams& G, std::string* src, int64_t* grid, int* block, int* smem, JitArgs* args) {
  constexpr int WARPS = 8;
  const int64_t M = G.M, K = G.K, N = G.N;
  if (M < 2 || M > 8 || K % 128 != 0 || (M > 1 && G.x_sm != G.K)) return false;
  const int XP = G.x_dt == KDT_F32 ? 3 : 1;
  if (!(G.x_dt == KDT_BF16 || G.x_dt == KDT_F32)) return false;
  const int64_t rowb = (K + 8) * 2;                   // padded shared row, bytes
  const int64_t stage_b = 8 * rowb, x_b = XP * 8 * rowb;
  const int NST = (int)std::min<int64_t>(4, (200 * 1024 - x_b) / stage_b);
  if (NST < 2) return false;
  *args = JitArgs{};
  const int kW = 0, kY = G.nseg, kS = 2 * G.nseg, kX = kS + 1;
  if (kX + 1 > JIT_MAXBUF) return false;
  auto put = [&](int k, const DPtr& p) {
    args->s[k] = p.slot;
    args->o[k] = p.off;
  };
  for (int i = 0; i < G.nseg; ++i) {
    put(kW + i, G.w[i]);
    put(kY + i, G.y[i]);
  }
  put(kS, G.status);
  put(kX, G.x);
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(sm_count(), (N + 7) / 8));
  const int64_t KW = K / WARPS, KS = KW / 16;  // columns and k-steps per warp
  std::ostringstream s;
  s << kPrelude << args_struct();
  s << gemv_mma_helpers();
  s << "__device__ __forceinline__ i64 stage_end(i64 r, i64 r1) {\n  i64 e = r + 8LL;\n  if (e > r1) e = r1;\n";
  for (int i = 0; i + 1 < G.nseg; ++i)
    s << "  if (r < " << G.seg_end[i] << "LL && e > " << G.seg_end[i] << "LL) e = " << G.seg_end[i] << "LL;\n";
  s << "  return e;\n}\n";
  auto seg_chain = [&](const std::string& row, const std::string& ind) {
    std::ostringstream c;
    c << ind << "int sg = 0; i64 lo = 0;\n";
    for (int i = 0; i + 1 < G.nseg; ++i)
      c << ind << "if (" << row << " >= " << G.seg_end[i] << "LL) { sg = " << i + 1 << "; lo = " << G.seg_end[i] << "LL; }\n";
    return c.str();
  };
  s << "extern \"C\" __global__ void __launch_bounds__(" << (WARPS + 1) * 32
    << ", 1) cljxla_fused_gemv(const u64* __restrict__ argtab, const JitArgs a) {\n";
  s << "  extern __shared__ __align__(1024) unsigned char dsm[];\n";
  s << "  __shared__ __align__(8) unsigned long long full_bar[" << NST << "], empty_bar[" << NST << "];\n";
  s << "  __shared__ float red[" << NST << "][8][8][8];\n";
  s << "  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;\n";
  s << "  const i64 r0 = (i64)" << N << "LL * blockIdx.x / gridDim.x, r1 = (i64)" << N << "LL * (blockIdx.x + 1) / gridDim.x;\n";
  s << "  unsigned* status = (unsigned*)" << base_expr(kS) << ";\n";
  s << "  const u32 stage0 = sa(dsm), xs0 = stage0 + " << (int64_t)NST * stage_b << "u;\n";
  s << "  if (threadIdx.x == 0) {\n    for (int i = 0; i < " << NST << "; ++i) { mb_init(sa(&full_bar[i]), 1u); mb_init(sa(&empty_bar[i]), "
    << WARPS << "u); }\n";
  s << "    asm volatile(\"fence.mbarrier_init.release.cluster;\" ::: \"memory\");\n  }\n  __syncthreads();\n";
  // producer: each weight row of a stage to its padded shared row, one mbarrier per stage
  s << "  if (warp == " << WARPS << ") {\n    if (lane != 0) return;\n    int st = 0;\n    bool ok = true;\n";
  s << "    for (i64 r = r0; r < r1; ++st) {\n      const int slot = st % " << NST << ";\n";
  s << "      if (st >= " << NST << " && !mb_wait(sa(&empty_bar[slot]), (u32)((st / " << NST << " - 1) & 1))) { ok = false; break; }\n";
  s << "      const i64 e = stage_end(r, r1);\n";
  s << seg_chain("r", "      ");
  s << "      const unsigned char* W = (const unsigned char*)";
  for (int i = 0; i + 1 < G.nseg; ++i) s << "(sg == " << i << " ? " << base_expr(kW + i) << " : ";
  s << base_expr(kW + G.nseg - 1);
  for (int i = 0; i + 1 < G.nseg; ++i) s << ")";
  s << ";\n";
  s << "      mb_expect(sa(&full_bar[slot]), (u32)((e - r) * " << K * 2 << "LL));\n";
  s << "      for (i64 q = r; q < e; ++q)\n        bulk_g2s(stage0 + (u32)slot * " << stage_b << "u + (u32)(q - r) * " << rowb
    << "u, W + (q - lo) * " << K * 2 << "LL, " << K * 2 << "u, sa(&full_bar[slot]));\n";
  s << "      r = e;\n    }\n    if (!ok) atomicOr(status, 4u);\n";
  s << "    for (int k = st - 1; k >= 0 && k >= st - " << NST << "; --k)\n";
  s << "      if (!mb_wait(sa(&full_bar[k % " << NST << "]), (u32)((k / " << NST << ") & 1))) atomicOr(status, 8u);\n";
  s << "    return;\n  }\n";
  // consumers: x as bf16 parts in padded rows (rows >= M zero)
  s << "  pdl_enter();\n  {\n    const char* X = " << base_expr(kX) << ";\n";
  s << "    for (int e = threadIdx.x; e < " << 8 * K << "; e += 256) {\n";
  s << "      const int m = e / " << K << ", k = e % " << K << ";\n";
  s << "      unsigned short p[3] = {0, 0, 0};\n";
  if (XP == 1) {
    s << "      if (m < " << M << ") p[0] = ((const unsigned short*)X)[(i64)m * " << K << " + k];\n";
  } else {
    s << "      if (m < " << M << ") {\n        const float q = ((const float*)X)[(i64)m * " << K << " + k];\n";
    s << "        p[0] = f2bf(q);\n        const float r1 = q - __uint_as_float((u32)p[0] << 16);\n";
    s << "        p[1] = f2bf(r1);\n        p[2] = f2bf(r1 - __uint_as_float((u32)p[1] << 16));\n      }\n";
  }
  s << "      for (int part = 0; part < " << XP << "; ++part)\n";
  s << "        *(unsigned short*)(dsm + " << (int64_t)NST * stage_b << " + part * " << 8 * rowb << " + m * " << rowb
    << " + k * 2) = p[part];\n    }\n  }\n  consumers_sync();\n";
  s << "  const u32 xa = xs0 + (u32)(g * " << rowb << " + (warp * " << KW << " + 2 * t) * 2);\n";
  s << "  const u32 wrow = (u32)((lane & 7) * " << rowb << " + (warp * " << KW << " + 8 * ((lane >> 3) & 1)) * 2);\n";
  s << "  int st = 0;\n  for (i64 r = r0; r < r1; ++st) {\n    const int slot = st % " << NST << ";\n";
  s << "    const i64 e = stage_end(r, r1);\n";
  s << "    bool bad = !mb_wait(sa(&full_bar[slot]), (u32)((st / " << NST << ") & 1));\n";
  s << "    bad = consumers_any(bad);\n    if (bad) { if (threadIdx.x == 0) atomicOr(status, 16u); break; }\n";
  s << "    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};\n";
  s << "    const u32 wb = stage0 + (u32)slot * " << stage_b << "u + wrow;\n";
  s << "#pragma unroll 4\n    for (int kk = 0; kk < " << KS << "; ++kk) {\n      u32 b0, b1;\n      ldsm_x2(wb + 32u * kk, b0, b1);\n";
  for (int part = 0; part < XP; ++part)
    s << "      mma16816(acc[kk & 1], lds32(xa + " << part * 8 * rowb << "u + 32u * kk), lds32(xa + " << part * 8 * rowb
      << "u + 32u * kk + 16u), b0, b1);\n";
  s << "    }\n    __syncwarp();\n    if (lane == 0) mb_arrive(sa(&empty_bar[slot]));\n";
  s << "    if (g < " << M << ") {\n      red[slot][warp][g][2 * t] = acc[0][0] + acc[1][0];\n"
       "      red[slot][warp][g][2 * t + 1] = acc[0][1] + acc[1][1];\n    }\n    consumers_sync();\n";
  s << "    if (threadIdx.x < " << M * 8 << ") {\n      const int m = threadIdx.x >> 3, n = threadIdx.x & 7;\n";
  s << "      const i64 row = r + n;\n      if (row < e) {\n        float v = 0.f;\n";
  s << "        for (int w = 0; w < " << WARPS << "; ++w) v += red[slot][w][m][n];\n";
  s << seg_chain("row", "        ");
  for (int i = 0; i < G.nseg; ++i) {
    const int64_t rows = G.seg_end[i] - (i ? G.seg_end[i - 1] : 0);
    s << "        if (sg == " << i << ") { char* Y = " << base_expr(kY + i) << "; "
      << store_stmt("Y", "(i64)m * " + std::to_string(rows) + "LL + (row - lo)", G.y_dt[i], "U(v)") << " }\n";
  }
  s << "      }\n    }\n    r = e;\n  }\n}\n";
  *src = s.str();
  *grid = ctas;
  *block = (WARPS + 1) * 32;
  *smem = (int)((int64_t)NST * stage_b + x_b);
  return true;
}

// Batched rows when x does not fit in shared memory whole (large K, or f32 x):
// each stage holds 8 weight rows x KC columns and the matching KC columns of
// the M rows of x (raw element type; f32 x is split into three bf16 parts when
// the fragments are built), so a tile of 8 rows takes K / KC stages whose
// partial products accumulate in the warps' registers.  The producer issues
// the weight copies of the first stages before the dependency wait and the x
// copies (x comes from the previous kernel) after it.
bool describe_gemv_mma_chunked(const GemvParams& G, std::string* src, int64_t* grid, int* block, int* smem,
                               JitArgs* args) {
  constexpr int WARPS = 8;
  const int64_t M = G.M, K = G.K, N = G.N;
  if (M < 2 || M > 8 || K % 128 != 0 || G.x_sm != G.K) return false;
  if (!(G.x_dt == KDT_BF16 || G.x_dt == KDT_F32)) return false;
  const int xes = G.x_dt == KDT_F32 ? 4 : 2;
  int64_t KC = 0;
  for (int64_t c = 128; c <= 2048 && c <= K; c += 128)
    if (K % c == 0) KC = c;
  if (KC == 0) return false;
  const int64_t NKC = K / KC;
  const int64_t wrowb = (KC + 8) * 2, xrowb = KC * xes + 16;
  const int64_t stage_b = ((8 * wrowb + M * xrowb) + 127) / 128 * 128;
  const int NST = (int)std::min<int64_t>(4, (200 * 1024) / stage_b);
  if (NST < 2) return false;
  *args = JitArgs{};
  const int kW = 0, kY = G.nseg, kS = 2 * G.nseg, kX = kS + 1;
  if (kX + 1 > JIT_MAXBUF) return false;
  auto put = [&](int k, const DPtr& p) {
    args->s[k] = p.slot;
    args->o[k] = p.off;
  };
  for (int i = 0; i < G.nseg; ++i) {
    put(kW + i, G.w[i]);
    put(kY + i, G.y[i]);
  }
  put(kS, G.status);
  put(kX, G.x);
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(sm_count(), (N + 7) / 8));
  const int64_t KW = KC / WARPS, KS = KW / 16;
  const int XP = xes == 4 ? 3 : 1;
  std::ostringstream s;
  s << kPrelude << args_struct();
  s << gemv_mma_helpers();
  s << "__device__ __forceinline__ void mb_expect_only(u32 a, u32 bytes) {\n"
       "  asm volatile(\"mbarrier.expect_tx.shared::cta.b64 [%0], %1;\" ::\"r\"(a), \"r\"(bytes) : \"memory\");\n}\n";
  s << "__device__ __forceinline__ i64 tile_end(i64 r, i64 r1) {\n  i64 e = r + 8LL;\n  if (e > r1) e = r1;\n";
  for (int i = 0; i + 1 < G.nseg; ++i)
    s << "  if (r < " << G.seg_end[i] << "LL && e > " << G.seg_end[i] << "LL) e = " << G.seg_end[i] << "LL;\n";
  s << "  return e;\n}\n";
  auto seg_chain = [&](const std::string& row, const std::string& ind) {
    std::ostringstream c;
    c << ind << "int sg = 0; i64 lo = 0;\n";
    for (int i = 0; i + 1 < G.nseg; ++i)
      c << ind << "if (" << row << " >= " << G.seg_end[i] << "LL) { sg = " << i + 1 << "; lo = " << G.seg_end[i] << "LL; }\n";
    return c.str();
  };
  s << "extern \"C\" __global__ void __launch_bounds__(" << (WARPS + 1) * 32
    << ", 1) cljxla_fused_gemv(const u64* __restrict__ argtab, const JitArgs a) {\n";
  s << "  extern __shared__ __align__(1024) unsigned char dsm[];\n";
  s << "  __shared__ __align__(8) unsigned long long full_bar[" << NST << "], empty_bar[" << NST << "];\n";
  s << "  __shared__ float red[8][8][8];\n";
  s << "  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;\n";
  s << "  const i64 r0 = (i64)" << N << "LL * blockIdx.x / gridDim.x, r1 = (i64)" << N << "LL * (blockIdx.x + 1) / gridDim.x;\n";
  s << "  unsigned* status = (unsigned*)" << base_expr(kS) << ";\n";
  s << "  const u32 stage0 = sa(dsm);\n";
  s << "  if (threadIdx.x == 0) {\n    for (int i = 0; i < " << NST << "; ++i) { mb_init(sa(&full_bar[i]), 1u); mb_init(sa(&empty_bar[i]), "
    << WARPS << "u); }\n";
  s << "    asm volatile(\"fence.mbarrier_init.release.cluster;\" ::: \"memory\");\n  }\n  __syncthreads();\n";
  // producer
  s << "  if (warp == " << WARPS << ") {\n    if (lane != 0) return;\n";
  s << "    const char* X = " << base_expr(kX) << ";\n";
  auto wcopies = [&](const std::string& ind) {
    std::ostringstream c;
    c << seg_chain("r", ind);
    c << ind << "const unsigned char* W = (const unsigned char*)";
    for (int i = 0; i + 1 < G.nseg; ++i) c << "(sg == " << i << " ? " << base_expr(kW + i) << " : ";
    c << base_expr(kW + G.nseg - 1);
    for (int i = 0; i + 1 < G.nseg; ++i) c << ")";
    c << ";\n";
    c << ind << "for (i64 q = r; q < e; ++q)\n" << ind << "  bulk_g2s(stage0 + (u32)slot * " << stage_b << "u + (u32)(q - r) * "
      << wrowb << "u, W + (q - lo) * " << K * 2 << "LL + (i64)kc * " << KC * 2 << "LL, " << KC * 2
      << "u, sa(&full_bar[slot]));\n";
    return c.str();
  };
  auto xcopies = [&](const std::string& ind) {
    std::ostringstream c;
    c << ind << "for (int m = 0; m < " << M << "; ++m)\n" << ind << "  bulk_g2s(stage0 + (u32)slot * " << stage_b << "u + "
      << 8 * wrowb << "u + (u32)m * " << xrowb << "u, X + ((i64)m * " << K << " + (i64)kc * " << KC << ") * " << xes
      << ", " << KC * xes << "u, sa(&full_bar[slot]));\n";
    return c.str();
  };
  // weights of the first stages before the dependency wait
  s << "    {\n      int st = 0;\n      for (i64 r = r0; r < r1 && st < " << NST << ";) {\n";
  s << "        const i64 e = tile_end(r, r1);\n";
  s << "        for (int kc = 0; kc < " << NKC << " && st < " << NST << "; ++kc, ++st) {\n";
  s << "          const int slot = st;\n";
  s << "          mb_expect_only(sa(&full_bar[slot]), (u32)((e - r) * " << KC * 2 << "LL));\n";
  s << wcopies("          ");
  s << "        }\n        r = e;\n      }\n    }\n";
  s << "    asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
  s << "    int st = 0;\n    bool ok = true;\n";
  s << "    for (i64 r = r0; r < r1 && ok;) {\n      const i64 e = tile_end(r, r1);\n";
  s << "      for (int kc = 0; kc < " << NKC << "; ++kc, ++st) {\n        const int slot = st % " << NST << ";\n";
  s << "        if (st >= " << NST << ") {\n";
  s << "          if (!mb_wait(sa(&empty_bar[slot]), (u32)((st / " << NST << " - 1) & 1))) { ok = false; break; }\n";
  s << "          mb_expect(sa(&full_bar[slot]), (u32)((e - r) * " << KC * 2 << "LL + " << M * KC * xes << "LL));\n";
  s << wcopies("          ");
  s << "        } else {\n          mb_expect(sa(&full_bar[slot]), " << M * KC * xes << "u);\n        }\n";
  s << xcopies("        ");
  s << "      }\n      r = e;\n    }\n    if (!ok) atomicOr(status, 4u);\n";
  s << "    for (int k = st - 1; k >= 0 && k >= st - " << NST << "; --k)\n";
  s << "      if (!mb_wait(sa(&full_bar[k % " << NST << "]), (u32)((k / " << NST << ") & 1))) atomicOr(status, 8u);\n";
  s << "    return;\n  }\n";
  // consumers
  s << "  pdl_enter();\n";
  s << "  const u32 wofs = (u32)((lane & 7) * " << wrowb << " + (warp * " << KW << " + 8 * ((lane >> 3) & 1)) * 2);\n";
  s << "  const u32 xofs = " << 8 * wrowb << "u + (u32)(g * " << xrowb << " + (warp * " << KW << " + 2 * t) * " << xes << ");\n";
  s << "  int st = 0;\n  bool bad = false;\n";
  s << "  for (i64 r = r0; r < r1 && !bad;) {\n    const i64 e = tile_end(r, r1);\n";
  s << "    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};\n";
  s << "    for (int kc = 0; kc < " << NKC << "; ++kc, ++st) {\n      const int slot = st % " << NST << ";\n";
  s << "      bad = consumers_any(!mb_wait(sa(&full_bar[slot]), (u32)((st / " << NST << ") & 1)));\n";
  s << "      if (bad) { if (threadIdx.x == 0) atomicOr(status, 16u); break; }\n";
  s << "      const u32 sb = stage0 + (u32)slot * " << stage_b << "u;\n";
  s << "#pragma unroll 4\n      for (int kk = 0; kk < " << KS << "; ++kk) {\n        u32 b0, b1;\n";
  s << "        ldsm_x2(sb + wofs + 32u * kk, b0, b1);\n";
  if (XP == 1) {
    s << "        const u32 a0 = g < " << M << " ? lds32(sb + xofs + 32u * kk) : 0u;\n";
    s << "        const u32 a2 = g < " << M << " ? lds32(sb + xofs + 32u * kk + 16u) : 0u;\n";
    s << "        mma16816(acc[kk & 1], a0, a2, b0, b1);\n";
  } else {
    s << "        float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;\n";
    s << "        if (g < " << M << ") {\n          const float2 u = lds64f(sb + xofs + 64u * kk), v = lds64f(sb + xofs + 64u * kk + 32u);\n";
    s << "          q0 = u.x; q1 = u.y; q2 = v.x; q3 = v.y;\n        }\n";
    s << "        for (int part = 0; part < 3; ++part) {\n";
    s << "          const u32 a0 = pack2(q0, q1), a2 = pack2(q2, q3);\n";
    s << "          mma16816(acc[kk & 1], a0, a2, b0, b1);\n";
    s << "          q0 -= lo_bf(a0); q1 -= hi_bf(a0); q2 -= lo_bf(a2); q3 -= hi_bf(a2);\n        }\n";
  }
  s << "      }\n      __syncwarp();\n      if (lane == 0) mb_arrive(sa(&empty_bar[slot]));\n    }\n";
  s << "    if (bad) break;\n";
  s << "    if (g < " << M << ") {\n      red[warp][g][2 * t] = acc[0][0] + acc[1][0];\n"
       "      red[warp][g][2 * t + 1] = acc[0][1] + acc[1][1];\n    }\n    consumers_sync();\n";
  s << "    if (threadIdx.x < " << M * 8 << ") {\n      const int m = threadIdx.x >> 3, n = threadIdx.x & 7;\n";
  s << "      const i64 row = r + n;\n      if (row < e) {\n        float v = 0.f;\n";
  s << "        for (int w = 0; w < " << WARPS << "; ++w) v += red[w][m][n];\n";
  s << seg_chain("row", "        ");
  for (int i = 0; i < G.nseg; ++i) {
    const int64_t rows = G.seg_end[i] - (i ? G.seg_end[i - 1] : 0);
    s << "        if (sg == " << i << ") { char* Y = " << base_expr(kY + i) << "; "
      << store_stmt("Y", "(i64)m * " + std::to_string(rows) + "LL + (row - lo)", G.y_dt[i], "U(v)") << " }\n";
  }
  s << "      }\n    }\n    r = e;\n  }\n}\n";
  *src = s.str();
  *grid = ctas;
  *block = (WARPS + 1) * 32;
  *smem = (int)((int64_t)NST * stage_b);
  return true;
}

bool describe_gemv_tma(const Launch& l, std::string* src, int64_t* grid, int* block, int* smem, JitArgs* args) {
  const bool fused = l.kind == K_GEMV_FUSED;
  const bool tail = l.kind == K_GEMV_TAIL;
  if (!(l.kind == K_GEMV || (fused && l.parts.size() == 1) || (tail && !l.parts.empty()))) return false;
  const GemvParams& G = *(const GemvParams*)l.blob.data();
  if (tail && (G.M != 1 || !jit_gemv_tail_ok(G))) return false;
  if (!G.has_status) return false;  // no status word: keep the plain kernel
  static const bool off = [] {
    const char* e = getenv("CLJXLA_B200_GEMV_TMA");
    return e && e[0] == '0';
  }();
  if (off) return false;
  // epilogue: an elementwise program over the GEMV's rows runs in each CTA once
  // its rows are done; with two equal segments a CTA takes the same rows of
  // both (gate and up of a GeGLU), so every element it computes is local
  const bool epi = !l.epi.empty();
  const bool paired = epi && G.nseg == 2;
  const int64_t EF = paired ? G.seg_end[0] : G.N;  // rows per pass
  const int NP = paired ? 2 : 1;
  if (epi && (tail || G.M != 1 || G.nseg > 2 || (paired && G.seg_end[1] != 2 * G.seg_end[0]) ||
              l.epi.size() != 1 || l.epi[0].kind != K_EW))
    return false;
  // group tails: row programs over whole groups of output rows
  const bool gt = !l.gtail.empty();
  if (gt && (tail || epi || G.M != 1)) return false;
  if (G.M >= 2 && !fused && !tail &&
      (describe_gemv_mma(G, src, grid, block, smem, args) || describe_gemv_mma_chunked(G, src, grid, block, smem, args)))
    return true;
  GemvGeometry geo;
  if (!gemv_tma_geometry(G, &geo)) return false;
  if (G.M > 1 && G.x_sm != G.K) return false;
  int npb = 0;
  *args = JitArgs{};
  if (fused) {
    const Launch& pro = l.parts[0];
    if (pro.kind == K_EW) npb = ((const EwParams*)pro.blob.data())->nin + ((const EwParams*)pro.blob.data())->nout;
    else if (pro.kind == K_ROWNORM) npb = ((const RowParams*)pro.blob.data())->nin + ((const RowParams*)pro.blob.data())->nout;
    else return false;
    int64_t g0;
    int b0, c0;
    if (!describe_one(pro, &g0, &b0, &c0, args)) return false;
  }
  const int kW = npb, kY = npb + G.nseg, kS = npb + 2 * G.nseg, kX = kS + 1, kT = kX + 1;
  if (kT + 1 > JIT_MAXBUF) return false;
  auto put = [&](int k, const DPtr& p) {
    args->s[k] = p.slot;
    args->o[k] = p.off;
  };
  for (int i = 0; i < G.nseg; ++i) {
    put(kW + i, G.w[i]);
    put(kY + i, G.y[i]);
  }
  put(kS, G.status);
  put(kX, G.x);
  if (tail || gt) put(kT, G.tail_ctr);
  constexpr int WARPS = 8;
  const int64_t M = G.M, K = G.K, N = G.N;
  const int WPR = geo.wpr, RPS = geo.rps, NST = geo.nstage;
  const int64_t KP = K / WPR;
  const int64_t ctas =
      std::max<int64_t>(1, std::min<int64_t>((int64_t)geo.ctas_per_sm * sm_count(), (N + RPS - 1) / RPS));
  const int xes = G.x_dt == KDT_F32 ? 4 : 2;
  const int stage_stride = (geo.stage_bytes + 1023) & ~1023;
  // tail: the last CTA to arrive runs the programs after the GEMV (the acquire
  // orders its loads after every CTA's rows; they read through L2)
  std::string tail_code;
  if (tail) {
    std::ostringstream t;
    const std::string ctr = "((unsigned*)" + base_expr(kT) + ")";
    t << "  {\n    __shared__ unsigned tail_last;\n    consumers_sync();\n";
    t << "    if (threadIdx.x == 0) {\n      unsigned old;\n";
    t << "      asm volatile(\"atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;\" : \"=r\"(old) : \"l\"(" << ctr
      << ") : \"memory\");\n";
    t << "      tail_last = old == gridDim.x - 1u;\n    }\n    consumers_sync();\n    if (tail_last) {\n";
    for (size_t i = 0; i < l.parts.size(); ++i)
      t << "      tail" << i << "(argtab, t.p[" << i << "], 0u, 1u);\n      consumers_sync();\n";
    t << "      if (threadIdx.x == 0) *" << ctr << " = 0u;  // ready for the next launch\n    }\n  }\n";
    tail_code = t.str();
  }
  // group tails: each row r of part i covers GEMV rows [G0, G1) of one segment;
  // a CTA that wrote some of them arrives on the group's counter, and the one
  // completing it (the count of CTAs whose row range meets [G0, G1) is fixed by
  // the partition r0 = N c / grid) runs the row and its epilogue; the rows are
  // read through L2 after the acquire
  struct GroupTail {
    int part, row, args, epi_args;
    int64_t g0, g1, target, rows, C;
  };
  std::vector<GroupTail> groups;
  if (gt) {
    int ai = 0;
    for (size_t i = 0; i < l.gtail.size(); ++i) {
      const Launch& q = l.gtail[i];
      const Launch& qb = q.kind == K_FUSED_DUS ? q.parts[0] : q;
      if (qb.kind != K_ROWNORM) return false;
      const RowParams& r = *(const RowParams*)qb.blob.data();
      int seg = -1;
      for (int j = 0; j < r.nin && seg < 0; ++j)
        for (int k = 0; k < G.nseg; ++k)
          if (r.in[j].p.slot == G.y[k].slot && r.in[j].p.off == G.y[k].off) seg = k;
      if (seg < 0) return false;
      const int64_t s0 = seg ? G.seg_end[seg - 1] : 0;
      if (G.seg_end[seg] - s0 != r.rows * r.C) return false;
      const int a = ai++;
      const int ea = q.epi.empty() ? -1 : ai++;
      for (int64_t row = 0; row < r.rows; ++row) {
        GroupTail g{(int)i, (int)row, a, ea, s0 + row * r.C, s0 + (row + 1) * r.C, 0, r.rows, r.C};
        for (int64_t c = 0; c < ctas; ++c) {
          const int64_t c0 = N * c / ctas, c1 = N * (c + 1) / ctas;
          if (c0 < g.g1 && g.g0 < c1) ++g.target;
        }
        groups.push_back(g);
      }
    }
    std::ostringstream t;
    const std::string ctr = "((unsigned*)" + base_expr(kT) + ")";
    t << "  {\n    __shared__ int gt_run;\n    __threadfence();  // this CTA's rows, before its arrivals\n"
         "    consumers_sync();\n";
    for (size_t gi = 0; gi < groups.size(); ++gi) {
      const GroupTail& g = groups[gi];
      t << "    if (r0 < " << g.g1 << "LL && " << g.g0 << "LL < r1) {\n";
      t << "      if (threadIdx.x == 0) {\n        unsigned old;\n";
      t << "        asm volatile(\"atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;\" : \"=r\"(old) : \"l\"(" << ctr << " + "
        << gi << ") : \"memory\");\n";
      t << "        gt_run = old == " << g.target - 1 << "u;\n      }\n      consumers_sync();\n      if (gt_run) {\n";
      t << "        gt" << g.part << "(argtab, t.p[" << g.args << "], " << g.row << "u, " << g.rows << "u);\n";
      if (g.epi_args >= 0)
        t << "        consumers_sync();\n        gte" << g.part << "(argtab, t.p[" << g.epi_args << "], " << g.row * g.C
          << "LL, " << (g.row + 1) * g.C << "LL);\n";
      t << "        consumers_sync();\n        if (threadIdx.x == 0) " << ctr << "[" << gi << "] = 0u;  // ready for the next launch\n";
      t << "      }\n      consumers_sync();\n    }\n";
    }
    t << "  }\n";
    tail_code = t.str();
  }
  std::ostringstream s;
  s << kPrelude << args_struct();
  s << R"G(__device__ __forceinline__ float bf_lo(u32 u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(u32 u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ u32 sa(const void* p) { return (u32)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mb_init(u32 a, u32 n) { asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(n)); }
__device__ __forceinline__ void mb_expect(u32 a, u32 bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(u32 a) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory"); }
__device__ __forceinline__ bool mb_try(u32 a, u32 parity) {
  u32 ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(a), "r"(parity) : "memory");
  return ok != 0;
}
// bounded wait: false after the iteration limit
__device__ __forceinline__ bool mb_wait(u32 a, u32 parity) {
  for (u32 i = 0; i < (1u << 22); ++i)
    if (mb_try(a, parity)) return true;
  return false;
}
__device__ __forceinline__ void bulk_g2s(u32 dst, const void* src, u32 bytes, u32 bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ uint4 lds16(u32 a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ bool consumers_any(bool p) {  // OR over the consumer warps (named barrier 1)
  u32 r;
  asm volatile("{\n\t.reg .pred q, o;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred o, 1, )G" << WARPS * 32 << R"G(, q;\n\tselp.u32 %0, 1, 0, o;\n\t}"
               : "=r"(r) : "r"((u32)p) : "memory");
  return r != 0;
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, )G" << WARPS * 32 << R"G(;" ::: "memory"); }
__device__ __forceinline__ float dot8(const uint4& w, const float* x) {
  float s = bf_lo(w.x) * x[0];
  s = fmaf(bf_hi(w.x), x[1], s); s = fmaf(bf_lo(w.y), x[2], s); s = fmaf(bf_hi(w.y), x[3], s);
  s = fmaf(bf_lo(w.z), x[4], s); s = fmaf(bf_hi(w.z), x[5], s); s = fmaf(bf_lo(w.w), x[6], s);
  s = fmaf(bf_hi(w.w), x[7], s);
  return s;
}
)G";
  if (xes == 2)
    s << "__device__ __forceinline__ void xs8(u32 a, float* o) {\n  const uint4 v = lds16(a);\n"
         "  o[0] = bf_lo(v.x); o[1] = bf_hi(v.x); o[2] = bf_lo(v.y); o[3] = bf_hi(v.y);\n"
         "  o[4] = bf_lo(v.z); o[5] = bf_hi(v.z); o[6] = bf_lo(v.w); o[7] = bf_hi(v.w);\n}\n";
  else
    s << "__device__ __forceinline__ void xs8(u32 a, float* o) {\n  const uint4 u = lds16(a), v = lds16(a + 16);\n"
         "  o[0] = __uint_as_float(u.x); o[1] = __uint_as_float(u.y); o[2] = __uint_as_float(u.z); o[3] = __uint_as_float(u.w);\n"
         "  o[4] = __uint_as_float(v.x); o[5] = __uint_as_float(v.y); o[6] = __uint_as_float(v.z); o[7] = __uint_as_float(v.w);\n}\n";
  if (fused) {
    BodyOpts bo;
    bo.block = WARPS * 32;
    bo.smem_out = G.pro_out;
    bo.sync = "consumers_sync()";  // the producer warp does not take part
    bo.row_cache = 12;             // a decode row on 256 threads: every input load in flight at once
    emit_body(s, l.parts[0], WARPS * 32, 1, "pro_body", bo);
  }
  // segment of a row: index, first row, weights
  auto seg_chain = [&](const std::string& row, const std::string& ind) {
    std::ostringstream c;
    c << ind << "int sg = 0; i64 lo = 0;\n";
    for (int i = 0; i + 1 < G.nseg; ++i)
      c << ind << "if (" << row << " >= " << G.seg_end[i] << "LL) { sg = " << i + 1 << "; lo = " << G.seg_end[i] << "LL; }\n";
    return c.str();
  };
  // end of the stage starting at row r: RPS rows, clipped to the CTA's range and the segment
  s << "__device__ __forceinline__ i64 stage_end(i64 r, i64 r1) {\n  i64 e = r + " << RPS << "LL;\n  if (e > r1) e = r1;\n";
  for (int i = 0; i + 1 < G.nseg; ++i)
    s << "  if (r < " << G.seg_end[i] << "LL && e > " << G.seg_end[i] << "LL) e = " << G.seg_end[i] << "LL;\n";
  s << "  return e;\n}\n";
  if (gt) {
    // the group-tail programs, bodies run by the 256 consumer threads of one CTA
    int np = 0;
    for (const Launch& q : l.gtail) np += 1 + (q.epi.empty() ? 0 : 1);
    s << "struct JitTail { JitArgs g; JitArgs p[" << np << "]; };\n";
    g_l2_loads = true;
    for (size_t i = 0; i < l.gtail.size(); ++i) {
      BodyOpts bo;
      bo.block = WARPS * 32;
      bo.sync = "consumers_sync()";
      bo.row_cache = 12;
      emit_body(s, l.gtail[i], WARPS * 32, 1, "gt" + std::to_string(i), bo);
      if (!l.gtail[i].epi.empty()) {
        BodyOpts be;
        be.block = WARPS * 32;
        be.sync = "consumers_sync()";
        be.ranged = true;
        emit_body(s, l.gtail[i].epi[0], WARPS * 32, 1, "gte" + std::to_string(i), be);
      }
    }
    g_l2_loads = false;
  }
  if (tail) {
    // the tail programs, each a body run by the 256 consumer threads of one CTA
    s << "struct JitTail { JitArgs g; JitArgs p[" << l.parts.size() << "]; };\n";
    g_l2_loads = true;
    for (size_t i = 0; i < l.parts.size(); ++i) {
      BodyOpts bo;
      bo.block = WARPS * 32;
      bo.sync = "consumers_sync()";
      bo.row_cache = 12;  // a decode row on 256 threads: its inputs stay in registers across phases
      emit_body(s, l.parts[i], WARPS * 32, 1, "tail" + std::to_string(i), bo);
    }
    g_l2_loads = false;
  }
  if (epi) {
    s << "struct JitEpi { JitArgs g; JitArgs e; };\n";
    BodyOpts bo;
    bo.block = WARPS * 32;
    bo.sync = "consumers_sync()";
    bo.ranged = true;
    emit_body(s, l.epi[0], WARPS * 32, 1, "epi_body", bo);
  }
  s << "extern \"C\" __global__ void __launch_bounds__(" << (WARPS + 1) * 32
    << ", " << geo.ctas_per_sm << ") cljxla_fused_gemv(const u64* __restrict__ argtab, const "
    << (tail || gt ? "JitTail t) {\n  const JitArgs& a = t.g;\n" : epi ? "JitEpi t) {\n  const JitArgs& a = t.g;\n" : "JitArgs a) {\n");
  s << "  extern __shared__ __align__(1024) unsigned char dsm[];\n";
  s << "  __shared__ __align__(8) unsigned long long full_bar[" << NST << "], empty_bar[" << NST << "];\n";
  s << "  __shared__ float red[" << NST << "][" << WARPS << "][" << M << "];\n";
  // rows of one CTA: with an epilogue, NP passes of at most ceil(EF / ctas) rows
  const int64_t max_rows = epi ? NP * ((EF + ctas - 1) / ctas) : (N + ctas - 1) / ctas;
  const bool late_sum = WPR > 1 && M == 1 && max_rows * WPR * 4 <= 16 * 1024;
  if (late_sum) s << "  __shared__ float rowpart[" << max_rows << "][" << WPR << "];\n";
  s << "  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;\n";
  if (epi)
    s << "  const i64 pa = (i64)" << EF << "LL * blockIdx.x / gridDim.x, pb = (i64)" << EF
      << "LL * (blockIdx.x + 1) / gridDim.x;\n";
  else
    s << "  const i64 r0 = (i64)" << N << "LL * blockIdx.x / gridDim.x, r1 = (i64)" << N << "LL * (blockIdx.x + 1) / gridDim.x;\n";
  // with an epilogue the row loops run once per pass over [pa, pb) + pass * EF
  const std::string pass_open = epi ? "  for (int pass = 0; pass < " + std::to_string(NP) +
                                          " && !quit; ++pass) {\n  const i64 r0 = pa + pass * " + std::to_string(EF) +
                                          "LL, r1 = pb + pass * " + std::to_string(EF) + "LL, rb = pass * (pb - pa);\n"
                                    : "";
  const std::string pass_close = epi ? "  }\n" : "";
  s << "  unsigned* status = (unsigned*)" << base_expr(kS) << ";\n";
  s << "  const u32 stage0 = sa(dsm), xsa = stage0 + " << (int64_t)NST * stage_stride << "u;\n";
  s << "  if (threadIdx.x == 0) {\n    for (int i = 0; i < " << NST << "; ++i) { mb_init(sa(&full_bar[i]), 1u); mb_init(sa(&empty_bar[i]), "
    << WARPS << "u); }\n";
  s << "    asm volatile(\"fence.mbarrier_init.release.cluster;\" ::: \"memory\");\n  }\n  __syncthreads();\n";
  // producer
  s << "  if (warp == " << WARPS << ") {\n    if (lane != 0) return;\n";
  s << "    int st = 0;\n    bool ok = true;\n";
  if (epi) s << "    bool quit = false;\n" << pass_open;
  s << "    for (i64 r = r0; r < r1; ++st) {\n      const int slot = st % " << NST << ";\n";
  s << "      if (st >= " << NST << " && !mb_wait(sa(&empty_bar[slot]), (u32)((st / " << NST << " - 1) & 1))) { ok = false; break; }\n";
  s << "      const i64 e = stage_end(r, r1);\n";
  s << seg_chain("r", "      ");
  s << "      const unsigned char* W = (const unsigned char*)";
  for (int i = 0; i + 1 < G.nseg; ++i) s << "(sg == " << i << " ? " << base_expr(kW + i) << " : ";
  s << base_expr(kW + G.nseg - 1);
  for (int i = 0; i + 1 < G.nseg; ++i) s << ")";
  s << ";\n";
  s << "      const u32 bytes = (u32)((e - r) * " << K * 2 << "LL);\n";
  s << "      mb_expect(sa(&full_bar[slot]), bytes);\n";
  s << "      bulk_g2s(stage0 + (u32)slot * " << stage_stride << "u, W + (r - lo) * " << K * 2 << "LL, bytes, sa(&full_bar[slot]));\n";
  s << "      r = e;\n    }\n";
  if (epi) s << "    quit = !ok;\n" << pass_close;
  s << "    if (!ok) atomicOr(status, 4u);\n";
  // drain: the copies of the last stages issued have landed before the CTA may end
  s << "    for (int k = st - 1; k >= 0 && k >= st - " << NST << "; --k)\n";
  s << "      if (!mb_wait(sa(&full_bar[k % " << NST << "]), (u32)((k / " << NST << ") & 1))) atomicOr(status, 8u);\n";
  s << "    return;\n  }\n";
  // consumers: x
  s << "  pdl_enter();\n";
  if (fused) {
    s << "  pro_body(argtab, a, 0u, 1u, (char*)(dsm + " << (int64_t)NST * stage_stride << "), blockIdx.x == 0);\n";
  } else {
    s << "  {\n    const char* X = " << base_expr(kX) << ";\n";
    if (M == 1 || G.x_sm == K)
      s << "    for (int i = threadIdx.x; i < " << M * K * xes / 16 << "; i += " << WARPS * 32
        << ") *(uint4*)(dsm + " << (int64_t)NST * stage_stride << " + 16 * i) = *(const uint4*)(X + 16 * i);\n";
    s << "  }\n";
  }
  s << "  consumers_sync();\n";
  s << "  const int rr = warp / " << WPR << ", part = warp % " << WPR << ";\n";
  // M = 1: x is the same for every row; each lane keeps its x vectors in registers
  const int NV = (M == 1 && (KP / 8 + 31) / 32 <= 12) ? (int)((KP / 8 + 31) / 32) : 0;
  if (NV > 0) {
    s << "  float xr[" << NV << "][8];\n#pragma unroll\n  for (int i = 0; i < " << NV << "; ++i) {\n";
    s << "    const int v = lane + 32 * i;\n";
    s << "    if (v < " << KP / 8 << ") xs8(xsa + (u32)(part * " << KP * xes << "LL) + " << 8 * xes << "u * v, xr[i]);\n";
    s << "    else for (int e = 0; e < 8; ++e) xr[i][e] = 0.f;\n  }\n";
  }
  s << "  int st = 0;\n";
  if (epi) s << "  bool quit = false;\n" << pass_open;
  s << "  for (i64 r = r0; r < r1; ++st) {\n    const int slot = st % " << NST << ";\n";
  s << "    const i64 e = stage_end(r, r1);\n";
  s << "    bool bad = !mb_wait(sa(&full_bar[slot]), (u32)((st / " << NST << ") & 1));\n";
  // one row split over WPR warps: with M = 1 the parts of each of the CTA's rows
  // wait in shared memory and are summed once after the loop (no barrier per stage)
  if (WPR > 1 && !late_sum) s << "    bad = consumers_any(bad);\n";
  s << "    if (bad) { if (threadIdx.x == 0) atomicOr(status, 16u); " << (epi ? "quit = true; " : "") << "break; }\n";
  s << "    const i64 row = r + rr;\n    const bool active = row < e;\n";
  s << "    float acc[" << M << "];\n#pragma unroll\n    for (int m = 0; m < " << M << "; ++m) acc[m] = 0.f;\n";
  s << "    if (active) {\n";
  s << "      const u32 wa = stage0 + (u32)slot * " << stage_stride << "u + (u32)((rr * " << K << "LL + part * " << KP
    << "LL) * 2);\n";
  s << "      const u32 xa = xsa + (u32)(part * " << KP * xes << "LL);\n";
  if (NV > 0) {  // one row: this lane's x vectors are in registers
    s << "#pragma unroll\n      for (int i = 0; i < " << NV << "; ++i) {\n        const int v = lane + 32 * i;\n";
    s << "        if (v < " << KP / 8 << ") acc[0] += dot8(lds16(wa + 16u * v), xr[i]);\n      }\n    }\n";
  } else {
    s << "#pragma unroll 4\n      for (int v = lane; v < " << KP / 8 << "; v += 32) {\n";
    s << "        const uint4 w = lds16(wa + 16u * v);\n";
    s << "#pragma unroll\n        for (int m = 0; m < " << M << "; ++m) {\n          float xv[8];\n";
    s << "          xs8(xa + (u32)(m * " << K * xes << "LL) + " << 8 * xes << "u * v, xv);\n";
    s << "          acc[m] += dot8(w, xv);\n        }\n      }\n    }\n";
  }
  s << "    __syncwarp();\n    if (lane == 0) mb_arrive(sa(&empty_bar[slot]));  // this warp is done with the stage\n";
  s << "#pragma unroll\n    for (int m = 0; m < " << M << "; ++m)\n";
  s << "      for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);\n";
  if (late_sum) {
    s << "    if (lane == 0 && active) rowpart[" << (epi ? "rb + " : "") << "row - r0][part] = acc[0];\n    r = e;\n  }\n";
    s << pass_close << "  consumers_sync();\n";
    if (epi) {  // the CTA's rows of every pass, v-th in pass order
      s << "  for (i64 v = threadIdx.x; v < " << NP << " * (pb - pa); v += " << WARPS * 32 << ") {\n";
      s << "    const i64 row = v < pb - pa ? pa + v : " << EF << "LL + pa + (v - (pb - pa));\n";
      s << "    float t = 0.f;\n    for (int q = 0; q < " << WPR << "; ++q) t += rowpart[v][q];\n";
    } else {
      s << "  for (i64 row = r0 + threadIdx.x; row < r1; row += " << WARPS * 32 << ") {\n";
      s << "    float t = 0.f;\n    for (int q = 0; q < " << WPR << "; ++q) t += rowpart[row - r0][q];\n";
    }
    s << seg_chain("row", "    ");
    for (int i = 0; i < G.nseg; ++i) {
      const int64_t rows = G.seg_end[i] - (i ? G.seg_end[i - 1] : 0);
      s << "    if (sg == " << i << ") { char* Y = " << base_expr(kY + i) << "; "
        << store_stmt("Y", "row - lo", G.y_dt[i], "U(t)") << " }\n";
      (void)rows;
    }
    s << "  }\n" << tail_code;
    // the epilogue over this CTA's elements [pa, pb): its GEMV inputs were
    // stored above by the CTA's own threads (ordered by the barrier)
    if (epi) s << "  consumers_sync();\n  if (!quit) epi_body(argtab, t.e, pa, pb);\n";
    s << "}\n";
    *src = s.str();
    *grid = ctas;
    *block = (WARPS + 1) * 32;
    *smem = NST * stage_stride + geo.x_bytes;
    return true;
  }
  if (WPR > 1) {
    s << "    if (lane == 0) for (int m = 0; m < " << M << "; ++m) red[slot][warp][m] = acc[m];\n";
    s << "    consumers_sync();\n";
    s << "    if (part == 0 && lane == 0 && active)\n      for (int q = 1; q < " << WPR << "; ++q)\n"
         "        for (int m = 0; m < " << M << "; ++m) acc[m] += red[slot][warp + q][m];\n";
  }
  s << "    if (active && part == 0 && lane == 0) {\n";
  s << seg_chain("row", "      ");
  for (int i = 0; i < G.nseg; ++i) {
    const int64_t rows = G.seg_end[i] - (i ? G.seg_end[i - 1] : 0);
    s << "      if (sg == " << i << ") { char* Y = " << base_expr(kY + i) << "; for (int m = 0; m < " << M << "; ++m) "
      << store_stmt("Y", "(i64)m * " + std::to_string(rows) + "LL + (row - lo)", G.y_dt[i], "U(acc[m])") << " }\n";
  }
  s << "    }\n    r = e;\n  }\n" << pass_close << tail_code;
  if (epi) s << "  consumers_sync();\n  if (!quit) epi_body(argtab, t.e, pa, pb);\n";
  s << "}\n";
  *src = s.str();
  *grid = ctas;
  *block = (WARPS + 1) * 32;
  *smem = NST * stage_stride + geo.x_bytes;
  return true;
}

void emit_body(std::ostringstream& s, const Launch& l, int block, int cluster, const std::string& fname,
               const BodyOpts& bo) {
  if (l.kind == K_FUSED_DUS) {
    BodyOpts b2 = bo;
    b2.dus = dus_stores_of(l);
    emit_body(s, l.parts[0], block, cluster, fname, b2);
    return;
  }
  if (l.kind == K_EW) emit_ew_body(s, *(const EwParams*)l.blob.data(), fname, bo);
  else emit_row_body(s, *(const RowParams*)l.blob.data(), block, cluster, fname, bo);
}

}  // namespace

bool jit_describe(const Launch& l, std::string* src, int64_t* grid, int* block, int* cluster,
                  std::vector<JitArgs>* args, int* smem) {
  args->clear();
  *smem = 0;
  if (l.kind == K_GEMV_FUSED || l.kind == K_GEMV || l.kind == K_GEMV_TAIL) {
    JitArgs a;
    *cluster = 1;
    if (!describe_gemv_tma(l, src, grid, block, smem, &a)) return false;
    args->push_back(a);
    for (const Launch& e : l.epi) {  // the epilogue program's buffers
      int64_t g;
      int b, c;
      JitArgs ea;
      if (!describe_one(e, &g, &b, &c, &ea)) return false;
      args->push_back(ea);
    }
    for (const Launch& q : l.gtail) {  // each group-tail program's buffers, then its epilogue's
      int64_t g;
      int b, c;
      JitArgs qa;
      if (!describe_one(q, &g, &b, &c, &qa)) return false;
      args->push_back(qa);
      for (const Launch& e : q.epi) {
        if (!describe_one(e, &g, &b, &c, &qa)) return false;
        args->push_back(qa);
      }
    }
    if (l.kind == K_GEMV_TAIL)
      for (const Launch& p : l.parts) {
        int64_t g;
        int b, c;
        JitArgs pa;
        if (!describe_one(p, &g, &b, &c, &pa) || c != 1) return false;
        args->push_back(pa);
      }
    return true;
  }
  if (l.kind == K_MULTI) {
    // one kernel, CTA ranges running the parts' programs in order
    std::vector<int64_t> grids;
    for (const Launch& p : l.parts) {
      int64_t g;
      int b, c;
      JitArgs a;
      if (!describe_one(p, &g, &b, &c, &a)) return false;
      auto base = [](const Launch& x) { return x.kind == K_FUSED_DUS ? x.parts[0].kind : x.kind; };
      if (!args->empty() && (c != *cluster || base(p) != base(l.parts[0]))) return false;
      *block = args->empty() ? b : std::max(*block, b);  // row programs run at the largest block
      *cluster = c;
      grids.push_back(g);
      args->push_back(a);
    }
    // a row program's epilogue (an elementwise program over the elements of
    // its rows, schedule.cc fuse_row_epilogues): its buffers follow the parts'
    std::vector<int> epi_arg(l.parts.size(), -1);
    for (size_t i = 0; i < l.parts.size(); ++i) {
      if (l.parts[i].epi.empty()) continue;
      if (*cluster != 1 || l.parts[i].kind != K_ROWNORM || grids[i] != ((const RowParams*)l.parts[i].blob.data())->rows)
        return false;
      int64_t g;
      int b, c;
      JitArgs ea;
      if (!describe_one(l.parts[i].epi[0], &g, &b, &c, &ea)) return false;
      epi_arg[i] = (int)args->size();
      args->push_back(ea);
    }
    std::ostringstream s;
    s << kPrelude << args_struct();
    s << "struct JitMulti { JitArgs p[" << args->size() << "]; };\n";
    for (size_t i = 0; i < l.parts.size(); ++i) {
      emit_body(s, l.parts[i], *block, *cluster, "part" + std::to_string(i));
      if (epi_arg[i] >= 0) {
        BodyOpts bo;
        bo.block = *block;
        bo.ranged = true;
        emit_body(s, l.parts[i].epi[0], *block, 1, "epi" + std::to_string(i), bo);
      }
    }
    s << "extern \"C\" __global__ void __launch_bounds__(" << *block
      << ") cljxla_fused_multi(const u64* __restrict__ argtab, const JitMulti a) {\n  pdl_enter();\n"
         "  unsigned b = blockIdx.x;\n";
    int64_t total = 0;
    for (size_t i = 0; i < grids.size(); ++i) {
      s << "  if (b < " << grids[i] << "u) {\n    part" << i << "(argtab, a.p[" << i << "], b, " << grids[i] << "u);\n";
      if (epi_arg[i] >= 0) {  // this CTA's row(s), now in memory, through the epilogue
        const int64_t C = ((const RowParams*)l.parts[i].blob.data())->C;
        s << "    __syncthreads();\n    epi" << i << "(argtab, a.p[" << epi_arg[i] << "], (i64)b * " << C << "LL, (i64)(b + 1) * "
          << C << "LL);\n";
      }
      s << "    return;\n  }\n  b -= " << grids[i] << "u;\n";
      total += grids[i];
    }
    s << "}\n";
    *grid = total;
    *src = s.str();
    return true;
  }
  JitArgs a;
  if (!describe_one(l, grid, block, cluster, &a)) return false;
  args->push_back(a);
  if (l.kind == K_EW) *src = jit_source_ew(*(const EwParams*)l.blob.data());
  else if (l.kind == K_ROWNORM) *src = jit_source_row(*(const RowParams*)l.blob.data(), *block, *cluster);
  else {
    std::ostringstream s;
    s << kPrelude << args_struct();
    emit_body(s, l, *block, *cluster, "body");
    const bool ew = l.parts[0].kind == K_EW;
    s << "extern \"C\" __global__ void __launch_bounds__(" << *block << ") " << (ew ? "cljxla_fused_ew" : "cljxla_fused_row")
      << "(const u64* __restrict__ argtab, const JitArgs a) {\n  pdl_enter();\n  body(argtab, a, blockIdx.x, gridDim.x);\n}\n";
    *src = s.str();
  }
  return true;
}

std::vector<std::string> jit_plan_sources(const Plan& p) {
  std::vector<std::string> out;
  for (const Launch& l : p.launches) {
    std::string s;
    int64_t g;
    int b = 0, c = 1;
    std::vector<JitArgs> a;
    int sm;
    if (jit_describe(l, &s, &g, &b, &c, &a, &sm)) out.push_back(std::move(s));
  }
  return out;
}

// ------------------------------------------------------------------ NVRTC
namespace {

struct Nvrtc {
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
  decltype(&nvrtcVersion) version = nullptr;
  bool ok = false;
};

Nvrtc& nvrtc() {
  static Nvrtc n;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"};
    void* h = nullptr;
    for (const char* nm : names)
      if ((h = dlopen(nm, RTLD_NOW | RTLD_LOCAL))) break;
    if (!h) return;
    n.create = (decltype(n.create))dlsym(h, "nvrtcCreateProgram");
    n.compile = (decltype(n.compile))dlsym(h, "nvrtcCompileProgram");
    n.log_size = (decltype(n.log_size))dlsym(h, "nvrtcGetProgramLogSize");
    n.log = (decltype(n.log))dlsym(h, "nvrtcGetProgramLog");
    n.cubin_size = (decltype(n.cubin_size))dlsym(h, "nvrtcGetCUBINSize");
    n.cubin = (decltype(n.cubin))dlsym(h, "nvrtcGetCUBIN");
    n.destroy = (decltype(n.destroy))dlsym(h, "nvrtcDestroyProgram");
    n.version = (decltype(n.version))dlsym(h, "nvrtcVersion");
    n.ok = n.create && n.compile && n.log_size && n.log && n.cubin_size && n.cubin && n.destroy;
  });
  return n;
}

std::mutex g_cache_mu;
std::map<std::string, void*> g_cache;  // source -> cudaKernel_t (nullptr: failed)

const char* const kNvrtcOpts[] = {"-arch=sm_100a", "-fmad=false", "--std=c++17", "-default-device"};

// On-disk cache of compiled fused kernels, so a process compiling a graph it
// (or an earlier process) compiled before skips NVRTC: one file per program,
// named by the SHA-256 of the NVRTC version, options and source.  Directory:
// CLJXLA_B200_CACHE_DIR, else $XDG_CACHE_HOME/cljxla_b200, else
// $HOME/.cache/cljxla_b200; CLJXLA_B200_CACHE_DIR=0 turns it off.
std::atomic<int64_t> g_disk_hits{0}, g_disk_misses{0};

std::string disk_cache_dir() {
  const char* e = getenv("CLJXLA_B200_CACHE_DIR");
  if (e && (!strcmp(e, "0") || !strcmp(e, "off"))) return "";
  std::string d;
  if (e && *e) d = e;
  else if (const char* x = getenv("XDG_CACHE_HOME")) d = std::string(x) + "/cljxla_b200";
  else if (const char* h = getenv("HOME")) d = std::string(h) + "/.cache/cljxla_b200";
  if (d.empty()) return "";
  for (size_t i = 1; i <= d.size(); ++i)  // mkdir -p
    if (i == d.size() || d[i] == '/') mkdir(d.substr(0, i).c_str(), 0755);
  return d;
}

std::string disk_cache_key(const std::string& src) {
  int major = 0, minor = 0;
  if (nvrtc().version) nvrtc().version(&major, &minor);
  std::string k = "nvrtc " + std::to_string(major) + "." + std::to_string(minor) + "\n";
  for (const char* o : kNvrtcOpts) k += std::string(o) + "\n";
  k += src;
  return sha256_hex(k.data(), k.size());
}

std::vector<char> disk_cache_get(const std::string& dir, const std::string& key) {
  std::vector<char> out;
  FILE* f = fopen((dir + "/" + key + ".cubin").c_str(), "rb");
  if (!f) return out;
  fseek(f, 0, SEEK_END);
  const long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  if (n > 0) {
    out.resize((size_t)n);
    if (fread(out.data(), 1, (size_t)n, f) != (size_t)n) out.clear();
  }
  fclose(f);
  return out;
}

void disk_cache_put(const std::string& dir, const std::string& key, const std::vector<char>& cubin) {
  // written under a unique name, then renamed: readers never see a partial file
  const std::string tmp = dir + "/" + key + ".tmp" + std::to_string((long)getpid()) + "_" +
                          std::to_string((unsigned long long)(uintptr_t)&cubin);
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return;
  const bool ok = fwrite(cubin.data(), 1, cubin.size(), f) == cubin.size();
  fclose(f);
  if (!ok || rename(tmp.c_str(), (dir + "/" + key + ".cubin").c_str()) != 0) remove(tmp.c_str());
}

// NVRTC -> cubin; empty on failure (the log goes to `log` when given)
std::vector<char> nvrtc_cubin(const std::string& src, std::string* log_out);

std::vector<char> to_cubin(const std::string& src, std::string* log_out) {
  const std::string dir = disk_cache_dir();
  std::string key;
  if (!dir.empty()) {
    key = disk_cache_key(src);
    std::vector<char> c = disk_cache_get(dir, key);
    if (!c.empty()) {
      ++g_disk_hits;
      return c;
    }
  }
  std::vector<char> c = nvrtc_cubin(src, log_out);
  if (!dir.empty() && !c.empty()) {
    ++g_disk_misses;
    disk_cache_put(dir, key, c);
  }
  return c;
}

std::vector<char> nvrtc_cubin(const std::string& src, std::string* log_out) {
  Nvrtc& n = nvrtc();
  if (!n.ok) return {};
  nvrtcProgram prog;
  if (n.create(&prog, src.c_str(), "fused.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) return {};
  nvrtcResult r = n.compile(prog, 4, kNvrtcOpts);
  if (r != NVRTC_SUCCESS) {
    size_t ls = 0;
    n.log_size(prog, &ls);
    std::string log(ls, '\0');
    n.log(prog, &log[0]);
    if (log_out) *log_out = log;
    if (getenv("CLJXLA_B200_JIT_LOG"))
      fprintf(stderr, "cljxla jit: compile failed:\n%s\n--- source ---\n%s\n", log.c_str(), src.c_str());
    n.destroy(&prog);
    return {};
  }
  size_t cs = 0;
  n.cubin_size(prog, &cs);
  std::vector<char> cubin(cs);
  n.cubin(prog, cubin.data());
  n.destroy(&prog);
  return cubin;
}

void* compile_one(const std::string& src) {
  std::vector<char> cubin = to_cubin(src, nullptr);
  if (cubin.empty()) return nullptr;
  cudaLibrary_t lib = nullptr;
  if (cudaLibraryLoadData(&lib, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  cudaKernel_t k = nullptr;
  // the entry point: the identifier before the parameter list of the extern "C" kernel
  std::string entry;
  const size_t at = src.rfind("extern \"C\" __global__");
  const size_t paren = at == std::string::npos ? std::string::npos : src.find('(', src.find("cljxla_fused", at));
  if (paren != std::string::npos) {
    size_t b = paren;
    while (b > 0 && (isalnum((unsigned char)src[b - 1]) || src[b - 1] == '_')) --b;
    entry = src.substr(b, paren - b);
  }
  if (entry.empty() || cudaLibraryGetKernel(&k, lib, entry.c_str()) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return (void*)k;  // the library stays loaded for the life of the process
}

}  // namespace

bool jit_gemv_tail_ok(const GemvParams& g) {
  if (!jit_enabled() || !g.has_status || g.M != 1) return false;
  if (const char* e = getenv("CLJXLA_B200_GEMV_TMA"))
    if (e[0] == '0') return false;
  GemvGeometry geo;
  return gemv_tma_geometry(g, &geo);
}

bool jit_tail_program_ok(const Launch& l) {
  int64_t g;
  int b, c;
  JitArgs a;
  const Launch& base = l.kind == K_FUSED_DUS && !l.parts.empty() ? l.parts[0] : l;
  // one CTA runs the tail: a single row (the decode norms), or an elementwise
  // program of at most two elements per thread; more serial work than that in
  // one CTA costs more than the kernel boundary it removes (measured: the head
  // norms, RoPE and GeGLU of a Gemma-3-4B layer as tails doubled the step time)
  if (base.kind == K_ROWNORM) {
    const RowParams& r = *(const RowParams*)base.blob.data();
    if (r.rows != 1 || r.C > 12 * 256) return false;
  } else if (base.kind == K_EW) {
    if (((const EwParams*)base.blob.data())->n > 512) return false;
  } else {
    return false;
  }
  return describe_one(l, &g, &b, &c, &a) && c == 1;
}

void jit_disk_cache_stats(int64_t* hits, int64_t* misses) {
  if (hits) *hits = g_disk_hits.load();
  if (misses) *misses = g_disk_misses.load();
}

int jit_check_sources(const std::vector<std::string>& sources, std::string* first_log) {
  if (!nvrtc().ok) return -1;
  std::map<std::string, int> uniq;
  for (const std::string& s : sources) uniq[s] = 1;
  if (const char* dir = getenv("CLJXLA_B200_DUMP_JIT")) {  // debugging aid: the distinct sources as files
    int k = 0;
    for (auto& kv : uniq) {
      std::string path = std::string(dir) + "/jit_" + std::to_string(k++) + ".cu";
      if (FILE* f = fopen(path.c_str(), "w")) {
        fwrite(kv.first.data(), 1, kv.first.size(), f);
        fclose(f);
      }
    }
  }
  int failed = 0;
  for (auto& kv : uniq) {
    std::string log;
    if (to_cubin(kv.first, &log).empty()) {
      if (!failed && first_log) *first_log = log + "\n--- source ---\n" + kv.first;
      ++failed;
    }
  }
  return failed;
}

bool jit_enabled() {
  const char* e = getenv("CLJXLA_B200_JIT");
  if (e && (e[0] == '0' || e[0] == 'f' || e[0] == 'F' || e[0] == 'n' || e[0] == 'N')) return false;
  return nvrtc().ok;
}

std::vector<void*> jit_compile(const std::vector<std::string>& sources) {
  std::vector<void*> out(sources.size(), nullptr);
  if (!jit_enabled()) return out;
  std::vector<std::string> todo;
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    std::map<std::string, int> seen;
    for (const std::string& s : sources)
      if (!g_cache.count(s) && !seen.count(s)) {
        seen[s] = 1;
        todo.push_back(s);
      }
  }
  std::vector<void*> got(todo.size(), nullptr);
  const unsigned hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  std::vector<std::thread> pool;
  std::mutex next_mu;
  size_t next = 0;
  for (unsigned t = 0; t < std::min<size_t>(hw, todo.size()); ++t)
    pool.emplace_back([&] {
      for (;;) {
        size_t i;
        {
          std::lock_guard<std::mutex> lk(next_mu);
          if (next >= todo.size()) return;
          i = next++;
        }
        got[i] = compile_one(todo[i]);
      }
    });
  for (auto& th : pool) th.join();
  std::lock_guard<std::mutex> lk(g_cache_mu);
  for (size_t i = 0; i < todo.size(); ++i) g_cache[todo[i]] = got[i];
  for (size_t i = 0; i < sources.size(); ++i) out[i] = g_cache[sources[i]];
  return out;
}

void jit_launch(void* kernel, int64_t grid, int block, int cluster, int smem, const uint64_t* argtab,
                const std::vector<JitArgs>& jargs, cudaStream_t s) {
  // a library kernel is device-independent; its shared-memory opt-in is per device
  if (smem > 0) ensure_smem_optin((const void*)kernel, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3((unsigned)block, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  // the parts' JitArgs are contiguous, which is the kernel's by-value parameter layout
  void* args[] = {(void*)&argtab, (void*)jargs.data()};
  CUDA_OK(cudaLaunchKernelExC(&cfg, (const void*)kernel, args));
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("CLJXLA_B200_PDL");
    return !(e && (e[0] == '0' || e[0] == 'f' || e[0] == 'F' || e[0] == 'n' || e[0] == 'N'));
  }();
  return on;
}

void launch_failed(cudaError_t e) { fail(E_INTERNAL, std::string("kernel launch failed: ") + cudaGetErrorString(e)); }

}  // namespace cljxla
