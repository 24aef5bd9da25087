// Compiled fused kernels.
//
// The planner describes every fused elementwise group (EwParams) and row
// region (RowParams) as a small register program.  The interpreting kernels
// (ew_kernel, row_kernel) run any such program, but pay ~100 instructions of
// dispatch per program step; on decode shapes, where each launch touches a
// few thousand elements, that dispatch latency is the whole kernel time.
// This module turns each program into CUDA C++ with the shapes, strides,
// element types and argument-table slots as constants, compiles it once per
// distinct program with NVRTC for sm_100a (-fmad=false so every op rounds
// exactly as printed, like the interpreter), and launches the compiled kernel
// in place of the interpreter.  Identical programs (the same op chain in every
// layer, differing only in argument-table slots) are generated once per slot
// pattern and cached for the life of the process.
//
// NVRTC is loaded at run time (libnvrtc.so.12 of the CUDA toolkit); without
// it, or if a program fails to compile, the interpreting kernel runs instead.
#pragma once

#include <string>
#include <vector>

#include "fast_kernels.h"
#include "planner.h"

namespace cljxla {

// Source of a compiled kernel (entry points cljxla_fused_ew / cljxla_fused_row,
// parameters: the argument table and the launch's JitArgs).
std::string jit_source_ew(const EwParams& p);
std::string jit_source_row(const RowParams& p, int block, int cluster);

// Launch geometry the generated row kernel expects.
void row_launch_shape(const RowParams& p, int* block, int* cluster, int64_t* grid);

// Source and launch geometry of the compiled replacement of an elementwise /
// row launch; false for launches that have none.
bool jit_describe(const Launch& l, std::string* src, int64_t* grid, int* block, int* cluster,
                  std::vector<JitArgs>* args, int* smem);

// Compiles the sources (in parallel, cached by text) and returns one kernel
// handle per source (nullptr where compilation failed or NVRTC is missing).
std::vector<void*> jit_compile(const std::vector<std::string>& sources);

bool jit_enabled();

// Host-only check: compiles the distinct sources to cubin (no device needed)
// and returns how many failed (-1: NVRTC not available); the first failure's
// log and source go to first_log.
int jit_check_sources(const std::vector<std::string>& sources, std::string* first_log);
// whether a decode GEMV compiles to the bulk-copy kernel that can carry a tail
// (one x row), and whether a launch can be one of its tail programs (a small
// elementwise / row program, with folded KV writes, run by one CTA)
bool jit_gemv_tail_ok(const GemvParams& g);
bool jit_tail_program_ok(const Launch& l);

// programs found in / added to the on-disk cache of compiled fused kernels by this process
void jit_disk_cache_stats(int64_t* hits, int64_t* misses);

// The sources prepare_jit would compile for a plan.
std::vector<std::string> jit_plan_sources(const Plan& p);

// Launches a compiled kernel: grid x block threads, thread-block clusters of
// `cluster` CTAs along x when cluster > 1, `smem` bytes of dynamic shared memory.
void jit_launch(void* kernel, int64_t grid, int block, int cluster, int smem, const uint64_t* argtab,
                const std::vector<JitArgs>& args, cudaStream_t s);

}  // namespace cljxla
