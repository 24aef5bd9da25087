// Fused row regions: normalisation / softmax shaped chains in one kernel.
//
// Printed norms (norm.clj:6-35) and softmax (attention.clj:357-360) decompose
// into an elementwise producer, a reduce along the last axis, a short chain
// of per-row scalar ops and a broadcast back into elementwise consumers.  The
// generic path runs that as 3-4 kernels with round trips through HBM; here a
// CTA owns one row: each phase streams the row's columns through the register
// program (recomputing earlier per-element values instead of storing them),
// ends in a block reduction, and the per-row scalar program runs before the
// next phase.  Every op keeps its printed element type: results are rounded
// exactly where the graph rounds them.
#include "ew_exec.cuh"

namespace cljxla {
namespace {

template <int BLOCK>
__global__ void __launch_bounds__(BLOCK) row_kernel(const __grid_constant__ RowParams P,
                                                   const uint64_t* __restrict__ argtab) {
  __shared__ float red_f[BLOCK / 32];
  __shared__ float bcast;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t row = blockIdx.x; row < P.rows; row += gridDim.x) {
    int64_t idx[CLJXLA_MAXR];
    {  // row multi-index over the leading dims
      int64_t rem = row;
      for (int d = P.rank - 2; d >= 0; --d) {
        idx[d] = rem % P.dims[d];
        rem /= P.dims[d];
      }
    }
    uint32_t R[RP_NREG];
    for (int ph = 0; ph < P.nphase; ++ph) {
      const RowPhase& Ph = P.ph[ph];
      float acc = Ph.red_kind == 0 ? 0.0f : -INFINITY;
      for (int64_t c = threadIdx.x; c < P.C; c += BLOCK) {
        idx[P.rank - 1] = c;
        for (int pc = Ph.lo; pc < Ph.hi; ++pc) ew_step(P.code[pc], R, idx, P.rank, P.in, argtab);
        if (Ph.red_reg >= 0) {
          float x = __uint_as_float(R[Ph.red_reg]);
          acc = Ph.red_kind == 0 ? acc + x : fmaxf(acc, x);
        }
        for (int o = 0; o < P.nout; ++o)
          if (!P.out[o].scalar && P.out[o].phase == ph)
            st_elem(dres(P.out[o].p, argtab), row * P.C + c, P.out[o].dt, R[P.out[o].reg]);
      }
      if (Ph.red_reg >= 0) {
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) {
          float o = __shfl_xor_sync(0xffffffffu, acc, s);
          acc = Ph.red_kind == 0 ? acc + o : fmaxf(acc, o);
        }
        if (lane == 0) red_f[warp] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
          float t = Ph.red_kind == 0 ? 0.0f : -INFINITY;
          for (int w = 0; w < BLOCK / 32; ++w) t = Ph.red_kind == 0 ? t + red_f[w] : fmaxf(t, red_f[w]);
          t = Ph.red_kind == 0 ? t + Ph.red_init : fmaxf(t, Ph.red_init);
          bcast = rnd(t, Ph.red_dt);
        }
        __syncthreads();
        R[Ph.red_dst] = __float_as_uint(bcast);
        __syncthreads();
      }
      idx[P.rank - 1] = 0;
      for (int pc = Ph.slo; pc < Ph.shi; ++pc) ew_step(P.code[pc], R, idx, P.rank, P.in, argtab);
    }
    if (threadIdx.x == 0)
      for (int o = 0; o < P.nout; ++o)
        if (P.out[o].scalar) st_elem(dres(P.out[o].p, argtab), row, P.out[o].dt, R[P.out[o].reg]);
  }
}

}  // namespace

void launch_row(const RowParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.rows == 0) return;
  int64_t g = p.rows < 65535 ? p.rows : 65535;
  // few rows (decode: one token) leave most SMs idle, so the row's columns are
  // spread over as many threads as a CTA holds to shorten each phase
  if (p.rows <= 296 && p.C >= 2048) row_kernel<1024><<<(int)g, 1024, 0, s>>>(p, argtab);
  else if (p.rows <= 296 && p.C >= 512) row_kernel<512><<<(int)g, 512, 0, s>>>(p, argtab);
  else if (p.C >= 1024) row_kernel<256><<<(int)g, 256, 0, s>>>(p, argtab);
  else if (p.C >= 256) row_kernel<128><<<(int)g, 128, 0, s>>>(p, argtab);
  else row_kernel<64><<<(int)g, 64, 0, s>>>(p, argtab);
}

}  // namespace cljxla
