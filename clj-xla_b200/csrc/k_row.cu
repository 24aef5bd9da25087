// Fused row regions: normalisation / softmax shaped chains in one kernel.
//
// Printed norms (norm.clj:6-35) and softmax (attention.clj:357-360) decompose
// into an elementwise producer, a reduce along the last axis, a short chain
// of per-row scalar ops and a broadcast back into elementwise consumers.  The
// generic path runs that as 3-4 kernels with round trips through HBM; here a
// row is owned by one CTA, or - when there are too few rows to fill the GPU
// (decode: one token) - by a thread-block cluster of up to 8 CTAs that split
// the row's columns and combine their partial reductions through distributed
// shared memory.  Each phase streams the columns through the register program
// (recomputing earlier per-element values instead of storing them), ends in a
// reduction, and the per-row scalar program runs before the next phase.  Every
// op keeps its printed element type: results are rounded exactly where the
// graph rounds them.  Reductions combine in a fixed order (warp tree, warps in
// order, cluster ranks in order), so results do not vary from run to run.
#include <cooperative_groups.h>

#include "common.h"
#include "ew_exec.cuh"

namespace cg = cooperative_groups;

namespace cljxla {
namespace {

template <int BLOCK, int CL>
__global__ void __launch_bounds__(BLOCK) row_kernel(const __grid_constant__ RowParams P,
                                                   const uint64_t* __restrict__ argtab) {
  pdl_enter();
  __shared__ float red_f[BLOCK / 32];
  __shared__ float bcast;
  __shared__ float cl_part[RP_MAXPH];  // this CTA's partial of each phase (read by the cluster)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned crank = CL > 1 ? cg::this_cluster().block_rank() : 0;
  const int64_t Cc = (P.C + CL - 1) / CL;
  const int64_t c0 = (int64_t)crank * Cc, c1 = min(P.C, c0 + Cc);
  const int64_t nrow_groups = gridDim.x / CL;
  for (int64_t row = blockIdx.x / CL; row < P.rows; row += nrow_groups) {
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
      for (int64_t c = c0 + threadIdx.x; c < c1; c += BLOCK) {
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
        float t = Ph.red_kind == 0 ? 0.0f : -INFINITY;
        if (threadIdx.x == 0)
          for (int w = 0; w < BLOCK / 32; ++w) t = Ph.red_kind == 0 ? t + red_f[w] : fmaxf(t, red_f[w]);
        if constexpr (CL > 1) {
          cg::cluster_group cluster = cg::this_cluster();
          if (threadIdx.x == 0) cl_part[ph] = t;
          cluster.sync();  // every CTA's partial of this phase is visible
          if (threadIdx.x == 0) {
            t = Ph.red_kind == 0 ? 0.0f : -INFINITY;
            for (int r = 0; r < CL; ++r) {
              float v = *cluster.map_shared_rank(&cl_part[ph], (unsigned)r);
              t = Ph.red_kind == 0 ? t + v : fmaxf(t, v);
            }
          }
        }
        if (threadIdx.x == 0) {
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
    if (threadIdx.x == 0 && crank == 0)
      for (int o = 0; o < P.nout; ++o)
        if (P.out[o].scalar) st_elem(dres(P.out[o].p, argtab), row, P.out[o].dt, R[P.out[o].reg]);
  }
  // peers may still be reading this CTA's partials
  if constexpr (CL > 1) cg::this_cluster().sync();
}

template <int BLOCK, int CL>
void launch_cl(const RowParams& p, const uint64_t* argtab, cudaStream_t s) {
  launch_k(row_kernel<BLOCK, CL>, dim3((unsigned)(p.rows * CL)), dim3(BLOCK), 0, s, CL, p, argtab);
}

template <int CL>
void launch_cluster(const RowParams& p, int64_t cols, const uint64_t* argtab, cudaStream_t s) {
  if (cols <= 32) launch_cl<32, CL>(p, argtab, s);
  else if (cols <= 64) launch_cl<64, CL>(p, argtab, s);
  else if (cols <= 128) launch_cl<128, CL>(p, argtab, s);
  else launch_cl<256, CL>(p, argtab, s);
}

int row_cluster_size(int64_t rows, int64_t C) {
  // split rows across a cluster only while the GPU has idle SMs and every CTA keeps >= 32 columns
  int cl = 1;
  while (cl < 8 && rows * cl * 2 <= 2 * 148 && C / (cl * 2) >= 32) cl *= 2;
  return cl;
}

}  // namespace

void launch_row(const RowParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.rows == 0) return;
  const int cl = row_cluster_size(p.rows, p.C);
  const int64_t cols = (p.C + cl - 1) / cl;
  if (cl == 8) launch_cluster<8>(p, cols, argtab, s);
  else if (cl == 4) launch_cluster<4>(p, cols, argtab, s);
  else if (cl == 2) launch_cluster<2>(p, cols, argtab, s);
  else {
    int64_t g = p.rows < 65535 ? p.rows : 65535;
    if (p.C >= 1024) launch_k(row_kernel<256, 1>, dim3((int)g), dim3(256), 0, s, 1, p, argtab);
    else if (p.C >= 256) launch_k(row_kernel<128, 1>, dim3((int)g), dim3(128), 0, s, 1, p, argtab);
    else launch_k(row_kernel<64, 1>, dim3((int)g), dim3(64), 0, s, 1, p, argtab);
  }
}

}  // namespace cljxla
