// POD parameter blocks shared by the planner (host) and the CUDA kernels.
//
// Device pointers that change from one execution to the next (the caller's
// argument buffers and the freshly allocated result buffers) are never baked
// into kernel parameters.  A DPtr names either a fixed device address
// (constants, the executable's scratch arena) or a slot of the per-executable
// argument table, which the executor refreshes with one small host->device copy
// before launching.  Kernel parameters therefore stay identical across calls,
// and the whole launch sequence of an executable can be captured once into a
// CUDA graph and replayed.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include <utility>

namespace cljxla {

#ifndef CLJXLA_MAXR
#define CLJXLA_MAXR 8
#endif

struct DPtr {
  int32_t slot;  // >= 0: argtab[slot] + off ; < 0: off is an absolute device address
  int32_t pad_;
  int64_t off;   // bytes
};

#ifdef __CUDACC__
__device__ __forceinline__ char* dres(const DPtr& p, const uint64_t* __restrict__ argtab) {
  return p.slot >= 0 ? (char*)(argtab[p.slot] + (uint64_t)p.off) : (char*)(uintptr_t)p.off;
}

// Programmatic dependent launch.  Every kernel of a plan is launched so that
// it may start while its predecessor in the stream is still running; before
// touching anything the predecessor writes it waits for the predecessor's
// completion (griddepcontrol.wait, a no-op for a normal launch), and only then
// lets its own successor launch.  A kernel can thus be resident and ready
// (and prefetch what does not depend on its predecessor, such as weights)
// when the previous kernel ends, instead of paying the launch latency after.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_trigger();
}
#endif

// Whether plan kernels are launched as programmatic dependents (env
// CLJXLA_B200_PDL, default on).
bool pdl_enabled();
[[noreturn]] void launch_failed(cudaError_t e);

// Launches `kernel` with the programmatic-dependent-launch attribute when
// enabled (cluster dimension `cluster` along x when > 1).
template <typename... KArgs, typename... Args>
void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int cluster,
              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) launch_failed(e);
}

// element type codes used on the device (same numbering as cljxla::DT)
enum : int32_t { KDT_F32 = 0, KDT_BF16, KDT_F16, KDT_F64, KDT_I32, KDT_I64, KDT_I8, KDT_I16, KDT_U8, KDT_U32, KDT_I1 };

// A strided view over a materialized buffer (strides in elements).
struct TView {
  DPtr p;
  int32_t dt;
  int32_t rank;
  int64_t shape[CLJXLA_MAXR];
  int64_t stride[CLJXLA_MAXR];
};

// ------------------------------------------------------------ elementwise
// A fused elementwise region is a small register program evaluated once per
// element of the loop shape.
enum EwOpc : uint8_t {
  EW_LOAD = 0, EW_IMM, EW_IOTA,
  EW_ADD, EW_SUB, EW_MUL, EW_DIV, EW_MAX, EW_MIN,
  EW_EXP, EW_TANH, EW_SQRT, EW_RSQRT, EW_SIN, EW_COS, EW_LOGISTIC, EW_NEG, EW_ABS,
  EW_CONVERT, EW_CMP, EW_SELECT,
};

constexpr int EW_MAXIN = 12;
constexpr int EW_MAXCODE = 64;
constexpr int EW_MAXOUT = 4;
constexpr int EW_NREG = 32;

struct EwIn {
  DPtr p;
  int32_t dt;
  int32_t sel_dim;              // >= 0: concatenate operand, valid for sel_lo <= idx[sel_dim] < sel_hi
  int64_t sel_lo, sel_hi;       // (loaded at idx[sel_dim] - sel_lo; elsewhere the load yields register b)
  int64_t stride[CLJXLA_MAXR];  // per loop dim, elements (0 = broadcast)
};

struct EwInstr {
  uint8_t op;
  uint8_t dt;    // result element type (rounding / int vs float semantics)
  uint8_t dst;
  uint8_t a, b, c;
  uint8_t aux;   // LOAD: input index; IOTA: dim; CMP: direction; CONVERT: source dt
  uint8_t aux2;  // CMP: operand dt
  float fimm;
  int32_t iimm;
};

struct EwOut {
  DPtr p;
  int32_t dt;
  int32_t reg;
};

struct EwParams {
  int64_t n;
  int32_t rank, nin, ncode, nout;
  int64_t dims[CLJXLA_MAXR];
  EwIn in[EW_MAXIN];
  EwInstr code[EW_MAXCODE];
  EwOut out[EW_MAXOUT];
};

// -------------------------------------------------------------- row fusion
// A fused row region: elementwise work over a loop shape F = [rows..., C]
// plus reductions along the last axis whose per-row results feed later
// elementwise work (normalisations, softmax).  One CTA handles a row; the
// program runs in phases separated by block-wide reductions.  Registers
// 0..RP_SREG0-1 hold per-element values (recomputed in each phase that needs
// them), registers RP_SREG0.. hold per-row scalars.
constexpr int RP_MAXIN = 12;
constexpr int RP_MAXCODE = 96;
constexpr int RP_MAXPH = 4;
constexpr int RP_MAXOUT = 6;
constexpr int RP_SREG0 = 32;
constexpr int RP_NREG = 48;

struct RowPhase {
  uint16_t lo, hi;     // per-element code of this phase: code[lo, hi)
  uint16_t slo, shi;   // per-row code run after this phase's reduction: code[slo, shi)
  int8_t red_reg;      // register reduced at the end of the phase (-1: none)
  uint8_t red_kind;    // 0 add, 1 max
  uint8_t red_dst;     // scalar register receiving the reduced value
  uint8_t red_dt;      // result type of the reduce (rounding)
  float red_init;      // printed init value (0 or -1e30)
};

struct RowOut {
  DPtr p;
  int32_t dt;
  int16_t reg;
  int8_t phase;        // per-element output: stored during this phase
  int8_t scalar;       // 1: per-row output, one value per row
};

struct RowParams {
  int64_t rows, C;
  int32_t rank, nin, nphase, nout;
  int64_t dims[CLJXLA_MAXR];  // F
  EwIn in[RP_MAXIN];
  RowPhase ph[RP_MAXPH];
  EwInstr code[RP_MAXCODE];
  RowOut out[RP_MAXOUT];
};

void launch_row(const RowParams& p, const uint64_t* argtab, cudaStream_t s);

// --------------------------------------------------------------- reduce
struct ReduceParams {
  TView in;               // full input view
  DPtr out;               // dense output (kept dims, row-major)
  int32_t out_dt;
  int32_t kind;           // 0 add, 1 max
  int32_t nkeep, nred;
  int64_t keep_shape[CLJXLA_MAXR], keep_stride[CLJXLA_MAXR];
  int64_t red_shape[CLJXLA_MAXR], red_stride[CLJXLA_MAXR];
  int64_t n_out, n_red;
  float init;
};

// ------------------------------------------------------------ copy / misc
struct CopyParams {      // dst[view] = convert(src[view]); same shape
  TView src, dst;
  int64_t n;
};

struct GatherParams {    // out[r, :] = table[clamp(idx[r]), :]
  DPtr table;
  int32_t table_dt;
  int32_t idx_dt;
  int64_t rows_table, row_len, table_row_stride;
  TView idx;             // index view (rank = number of rows' dims), one index per row
  DPtr out;
  int64_t n_rows;
};

struct DusParams {       // out = operand with update written at clamped starts
  TView operand;         // same shape as out
  TView update;
  DPtr out;              // dense
  int32_t rank;
  int32_t dt;
  int64_t out_shape[CLJXLA_MAXR];
  int64_t upd_shape[CLJXLA_MAXR];
  // start index per dim: immediate or scalar device value
  int64_t start_imm[CLJXLA_MAXR];
  DPtr start_ptr[CLJXLA_MAXR];
  int32_t start_dt[CLJXLA_MAXR];
  int32_t start_is_ptr[CLJXLA_MAXR];
  int64_t n;
  int32_t in_place;      // operand and out alias: only the update window is written
  int32_t has_undo;      // in place over a caller's buffer: save the old window first
  DPtr undo;             // [int64 starts[8]] + old window values (undo record)
};

// Restores a saved window (an undo record) into a buffer: versioned in-place
// dynamic_update_slice, see runtime.h.
void launch_undo_apply(void* dst, const void* undo, int rank, const int64_t* out_shape, const int64_t* upd_shape,
                       int dt, cudaStream_t s);

// Holds the stream for about `ns` nanoseconds (one thread sleeping on the
// global timer, at most a fixed number of rounds).  Profiling enqueues it in
// front of a step so that the step's launches run back to back on the device
// instead of at the host's launch rate.
void launch_stream_hold(int64_t ns, cudaStream_t s);

// ------------------------------------------------------------------ GEMM
// C[b][m][n] = sum_k A[b][m][k] * B[b][k][n]; A/B strided, C dense row-major.
struct GemmParams {
  DPtr a, b, c;
  int32_t a_dt, b_dt, c_dt, pad_;
  int64_t batch, M, N, K;
  int64_t a_sb, a_sm, a_sk;
  int64_t b_sb, b_sk, b_sn;
  int64_t c_sb;  // = M*N for dense C
};

// launchers (argtab = device pointer of the executable's argument table)
void launch_ew(const EwParams& p, const uint64_t* argtab, cudaStream_t s);
void launch_reduce(const ReduceParams& p, const uint64_t* argtab, cudaStream_t s);
void launch_copy(const CopyParams& p, const uint64_t* argtab, cudaStream_t s);
void launch_gather(const GatherParams& p, const uint64_t* argtab, cudaStream_t s);
void launch_dus(const DusParams& p, const uint64_t* argtab, cudaStream_t s);
void launch_gemm(const GemmParams& p, const uint64_t* argtab, cudaStream_t s);

}  // namespace cljxla
