// Compiles a parsed graph into a launch plan for the B200.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "ir.h"
#include "kernels.h"

namespace cljxla {

enum KernelKind : int {
  K_EW = 0, K_REDUCE, K_COPY, K_GATHER, K_DUS, K_GEMM,
  K_GEMV, K_ATTN_DECODE, K_ATTN_COMBINE, K_ROWNORM, K_GEMM_TC,
  K_MULTI,  // independent compiled fused kernels merged into one launch (parts)
  K_ALLREDUCE,  // tensor-parallel sum over the client's NCCL communicator
  K_GEMV_FUSED,  // compiled GEMV whose x is computed in each CTA by its producer's program (parts[0])
  K_FUSED_DUS,   // elementwise / row program (parts[0]) that also writes its output into KV windows (parts[1..], K_DUS)
  K_ARGMAX,      // the printed in-graph argmax as one kernel (k_argmax.cu)
  K_GEMV_TAIL,   // compiled GEMV whose last CTA to finish then runs the small programs after it (parts)
  K_NUM_KINDS
};
const char* kernel_kind_name(int k);

// all_reduce (sum, or elementwise max) of `count` elements of type dt from src
// into dst; both in the scratch arena, whose addresses are fixed for the
// executable's life, so the collective can be captured into the CUDA graph.
struct AllReduceParams {
  DPtr src, dst;
  int64_t count;
  int32_t dt, ranks;
  int32_t reduce, pad_;  // RED_ADD or RED_MAX
};

// Buffers of a compiled fused kernel, passed by value at launch: buffer k is
// argument-table slot s[k] plus byte offset o[k] (s[k] < 0: o[k] is the address).
constexpr int JIT_MAXBUF = 24;
constexpr int JIT_MAXPARTS = 8;  // programs merged into one launch at most
struct JitArgs {
  int32_t s[JIT_MAXBUF];
  int32_t pad;
  int64_t o[JIT_MAXBUF];
};

struct Launch {
  int kind = 0;
  std::vector<uint8_t> blob;  // the kernel's POD parameter block
  std::string label;          // for profiling: which graph values it produces
  int64_t algo_bytes = 0;     // algorithmic HBM bytes (roofline accounting)
  int64_t algo_flops = 0;
  // compiled replacement of an interpreted elementwise / row launch (jit.h);
  // null: the interpreting kernel runs
  void* jit_fn = nullptr;
  int64_t jit_grid = 0;
  int jit_block = 0, jit_cluster = 1;
  int jit_smem = 0;  // dynamic shared memory bytes
  std::vector<JitArgs> jit_args;  // one per program (several for K_MULTI)
  std::vector<Launch> parts;      // K_MULTI: the merged launches, in order
  // K_GEMV / K_GEMV_FUSED: an elementwise program over the GEMV's rows that each
  // CTA runs on its own rows once they are done (a GeGLU over paired gate / up
  // segments); not compiled: it runs as its own launch after the GEMV
  std::vector<Launch> epi;
  // K_GEMV / K_GEMV_FUSED (one row of x): row programs over the GEMV's output
  // rows, each row (a group of GEMV rows) run by the CTA that completes it
  // (per-group arrival counters in GemvParams::tail_ctr); not compiled: they
  // run as their own launches after the GEMV
  std::vector<Launch> gtail;
};

struct TensorSpec {
  DT dt;
  std::vector<int64_t> shape;
  int64_t bytes() const { return numel(shape) * (int64_t)dt_size(dt); }
};

struct PlanOptions {
  bool fuse = true;          // elementwise fusion (off: one kernel per op, for debugging)
  bool fast_kernels = true;  // specialised GEMV / attention / tcgen05 paths
  bool kv_in_place = false;  // dynamic_update_slice results alias their operand storage
};

// A dynamic_update_slice executed in place over the storage of the caller's
// argument `param`, producing result `out` (KV-cache update).  Before writing,
// the kernel saves the window's old values into an undo record whose device
// address comes from argument-table slot `undo_slot`.
struct InplaceDus {
  int out = -1, param = -1, undo_slot = -1;
  int rank = 0;
  DT dt = DT::BF16;
  int64_t out_shape[CLJXLA_MAXR] = {}, upd_shape[CLJXLA_MAXR] = {};
  int64_t undo_bytes = 0;
};

// A TMA tensor map the executor encodes (host side) into the executable's
// tensor-map table whenever the operand's address changes: a 2-D bf16 view
// `base` of `outer` rows x `inner` elements, `row_bytes` apart, copied in
// boxes of box_outer x box_inner.
struct TmapSpec {
  DPtr base;
  int64_t inner = 0, outer = 0, row_bytes = 0;
  int box_inner = 0, box_outer = 0;
};

struct Plan {
  std::string name;
  std::vector<InplaceDus> inplace;
  // tensor maps (128 bytes each) followed by one 4-byte status word that
  // kernels with bounded waits set on a timeout; argument-table slot tmap_slot()
  std::vector<TmapSpec> tmaps;
  std::vector<TensorSpec> params, outs;
  std::vector<Launch> launches;
  int64_t arena_bytes = 0;
  std::vector<uint8_t> const_blob;  // uploaded once; DPtr slot = const_slot()
  // outs[i] may alias param alias_param[i] (in-place dynamic_update_slice), else -1
  std::vector<int> out_alias_param;
  int n_nodes = 0, n_live = 0, n_fused_groups = 0;
  int n_mask_computed = 0;  // attention launches whose mask is computed in the kernel, not read
  int n_jit_missing = 0;  // launches with a compiled form that did not compile (interpreting fallback runs)
  std::vector<int64_t> tmp_offsets;  // arena offset of each scratch buffer
  std::vector<int64_t> tmp_bytes;    // size of each scratch buffer
  // argument table layout: [params][outputs][undo records][constant blob][scratch buffers][tensor-map table]
  int dyn_slots() const { return (int)(params.size() + outs.size() + inplace.size()); }
  int const_slot() const { return dyn_slots(); }
  int tmp_slot0() const { return const_slot() + 1; }
  int tmap_slot() const { return tmp_slot0() + (int)tmp_offsets.size(); }
  bool needs_status = false;  // kernels with bounded waits that report through the status word
  bool has_table() const { return !tmaps.empty() || needs_status; }
  int64_t tmap_table_bytes() const { return has_table() ? 128 * (int64_t)tmaps.size() + 128 : 0; }
  int argtab_size() const { return tmap_slot() + (has_table() ? 1 : 0); }
};

std::unique_ptr<Plan> build_plan(const Graph& g, const PlanOptions& opt);

// Re-levels the launch list by the memory each launch touches and merges
// independent compiled fused kernels of one launch shape (schedule.cc).
void schedule_and_merge(Plan& p);

// Moves the elementwise program consuming a decode GEMV's rows element by
// element (the GeGLU after the gate / up projection) into the GEMV as an
// epilogue each CTA runs on its own rows (schedule.cc).
void fuse_gemv_epilogues(Plan& p);

// Moves the row programs that read a one-row GEMV's output by whole rows (the
// per-head q / k norms with their RoPE epilogue, the v norm) into the GEMV:
// the CTA that completes a row's GEMV rows runs that row (schedule.cc).
void fuse_gemv_group_tails(Plan& p);

// Moves an elementwise program that reads a row program's outputs only within
// each element's own row (RoPE after the per-head norms) into the row program's
// launch, run by the CTA of each row right after the row (schedule.cc).
void fuse_row_epilogues(Plan& p);

// Appends the small compiled programs that directly follow a decode GEMV to it
// as a tail its last CTA runs (K_GEMV_TAIL), removing their kernel boundaries
// (schedule.cc).
void fuse_gemv_tails(Plan& p);

// Generates and compiles the fused elementwise / row launches of a plan
// (no-op when runtime compilation is unavailable or disabled).
void prepare_jit(Plan& p);

// Dispatches one launch record (argtab: device pointer of the argument table).
void run_launch(const Launch& l, const uint64_t* argtab, cudaStream_t s);
void run_fast_launch(const Launch& l, const uint64_t* argtab, cudaStream_t s);

// Host-side bounds verification of every launch (throws INTERNAL on a violation).
void verify_plan(const Plan& p);

}  // namespace cljxla
