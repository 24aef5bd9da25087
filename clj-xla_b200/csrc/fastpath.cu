// Dispatch for the specialised kernels (decode GEMV, fused attention, row
// norms, tcgen05 GEMM).  Each kernel family lives in its own file and
// registers a launcher here.
#include "planner.h"

namespace cljxla {

void run_fast_launch(const Launch& l, const uint64_t* argtab, cudaStream_t s) {
  (void)argtab;
  (void)s;
  fail(E_INTERNAL, std::string("no launcher for kernel kind ") + kernel_kind_name(l.kind));
}

}  // namespace cljxla

namespace cljxla {
void verify_fast_launch(const Plan& p, const Launch& l) {
  (void)p;
  fail(E_INTERNAL, std::string("no bounds verifier for kernel kind ") + kernel_kind_name(l.kind));
}
}  // namespace cljxla
