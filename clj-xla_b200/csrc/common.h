// Shared definitions for libcljxla_b200: element types, status, small helpers.
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

namespace cljxla {

// Element types of the printed StableHLO subset (stablehlo.clj:6-7, plus i1 for
// compare results).
enum class DT : uint8_t { F32 = 0, BF16, F16, F64, I32, I64, I8, I16, U8, U32, I1, INVALID };

inline size_t dt_size(DT t) {
  switch (t) {
    case DT::F32: case DT::I32: case DT::U32: return 4;
    case DT::BF16: case DT::F16: case DT::I16: return 2;
    case DT::F64: case DT::I64: return 8;
    case DT::I8: case DT::U8: case DT::I1: return 1;
    default: return 0;
  }
}
inline bool dt_is_float(DT t) { return t == DT::F32 || t == DT::BF16 || t == DT::F16 || t == DT::F64; }
inline bool dt_is_int(DT t) { return !dt_is_float(t) && t != DT::INVALID; }

const char* dt_name(DT t);
DT dt_from_name(const std::string& s);
DT dt_from_pjrt(int pjrt_type);
int dt_to_pjrt(DT t);

// Errors raised inside the library; converted to PJRT_Error at the C boundary.
struct Error : std::runtime_error {
  int code;  // PJRT_Error_Code
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
[[noreturn]] void fail(int code, const std::string& msg);
inline void check(bool cond, int code, const std::string& msg) {
  if (!cond) fail(code, msg);
}
enum { E_INVALID = 3, E_NOT_FOUND = 5, E_OOM = 8, E_PRECOND = 9, E_UNIMPLEMENTED = 12, E_INTERNAL = 13 };

#define CUDA_OK(expr)                                                                  \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess)                                                             \
      ::cljxla::fail(_e == cudaErrorMemoryAllocation ? ::cljxla::E_OOM : ::cljxla::E_INTERNAL, \
                     std::string("CUDA error ") + cudaGetErrorString(_e) + " at " + __FILE__ + ":" + \
                         std::to_string(__LINE__));                                   \
  } while (0)

constexpr int MAXR = 8;  // max tensor rank handled by the kernels

inline int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  return n;
}
std::string shape_str(const std::vector<int64_t>& s);

// Library-wide counters (read through the C ABI).
struct Counters {
  int64_t kernel_launches = 0;
  int64_t executions = 0;
  int64_t graph_launches = 0;
};
Counters& counters();

// Facts about the current device, kept per device ordinal because a process
// may drive clients on several GPUs: its SM count (148 on B200), and the
// opt-in to more than 48 KB of dynamic shared memory, which
// cudaFuncSetAttribute applies to the current device only and is therefore
// recorded per (kernel, device).  Both throw Error on a CUDA failure.
int device_sm_count();
void ensure_smem_optin(const void* kernel, int bytes);

}  // namespace cljxla
