// Dispatch and bounds verification for the specialised kernels.
#include "fast_kernels.h"

namespace cljxla {

void run_fast_launch(const Launch& l, const uint64_t* argtab, cudaStream_t s) {
  switch (l.kind) {
    case K_GEMV: launch_gemv(*(const GemvParams*)l.blob.data(), argtab, s); break;
    case K_ATTN_DECODE: launch_attention(*(const AttnParams*)l.blob.data(), argtab, s); break;
    case K_ATTN_COMBINE: launch_attention_combine(*(const AttnParams*)l.blob.data(), argtab, s); break;
    case K_GEMM_TC: launch_tc_gemm(*(const TcGemmParams*)l.blob.data(), argtab, s); break;
    case K_ARGMAX: launch_argmax(*(const ArgmaxParams*)l.blob.data(), argtab, s); break;
    default: fail(E_INTERNAL, std::string("no launcher for kernel kind ") + kernel_kind_name(l.kind));
  }
}

void verify_fast_launch_impl(const Plan& p, const Launch& l, const RegionFn& region) {
  switch (l.kind) {
    case K_GEMV: case K_GEMV_FUSED: case K_GEMV_TAIL: verify_gemv(p, l, region); break;
    case K_ATTN_DECODE: case K_ATTN_COMBINE: verify_attention(l, region); break;
    case K_GEMM_TC: {
      const TcGemmParams& t = *(const TcGemmParams*)l.blob.data();
      if (t.tmap_a_index < 0 || t.tmap_b_index < 0 || t.tmap_a_index >= (int)p.tmaps.size() ||
          t.tmap_b_index >= (int)p.tmaps.size() || t.tmap_a.slot != p.tmap_slot())
        fail(E_INTERNAL, "tensor-core GEMM tensor maps not placed");
      verify_tc_gemm(t, region);
      break;
    }
    case K_ARGMAX: verify_argmax(*(const ArgmaxParams*)l.blob.data(), region); break;
    default: fail(E_INTERNAL, std::string("no bounds verifier for kernel kind ") + kernel_kind_name(l.kind));
  }
}

}  // namespace cljxla
