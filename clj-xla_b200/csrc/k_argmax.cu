// Greedy-sampling argmax of logits rows in one kernel.
//
// Replaces the printed in-graph argmax of tensor.clj:519-532 (reduce_max of
// the row, compare EQ against its broadcast, convert to i32, multiply by the
// iota literal, reduce_max of that), which as generic kernels is a row
// reduction, an elementwise pass writing an i32 index array and a one-block
// integer reduction over 262,144 entries.  Here each row is split over
// several CTAs; every thread keeps (value, index) with the printed tie rule
// (equal values: the highest index wins), the CTA reduces through shuffles and
// shared memory, and the last CTA of a row to arrive combines the CTAs'
// pairs.  The logits are read once.  A row whose values are all NaN gives
// index 0 (the printed graph's result there); with some NaN values this
// kernel ignores them, where the printed graph's NaN maximum would also give 0.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fast_kernels.h"

namespace cljxla {
namespace {

constexpr int AM_THREADS = 256;

__device__ __forceinline__ float am_load(const char* base, int64_t i, int dt) {
  if (dt == KDT_F32) return ((const float*)base)[i];
  if (dt == KDT_BF16) return __uint_as_float((uint32_t)((const uint16_t*)base)[i] << 16);
  return __half2float(((const __half*)base)[i]);
}

// (v, i) beats (bv, bi): larger value, or equal value and larger index
__device__ __forceinline__ void am_take(float v, int64_t i, float& bv, int64_t& bi) {
  if (v > bv || (v == bv && i > bi)) {
    bv = v;
    bi = i;
  }
}

__device__ __forceinline__ void am_warp(float& bv, int64_t& bi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t i = __shfl_xor_sync(0xffffffffu, bi, o);
    am_take(v, i, bv, bi);
  }
}

__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(const __grid_constant__ ArgmaxParams P,
                                                            const uint64_t* __restrict__ argtab) {
  pdl_enter();
  __shared__ float s_v[AM_THREADS / 32];
  __shared__ int64_t s_i[AM_THREADS / 32];
  __shared__ int s_last;
  const int64_t row = blockIdx.y;
  int64_t off = 0, rem = row;
  for (int d = P.in.rank - 2; d >= 0; --d) {
    off += (rem % P.in.shape[d]) * P.in.stride[d];
    rem /= P.in.shape[d];
  }
  const char* base = dres(P.in.p, argtab);
  const int64_t s_last_dim = P.in.stride[P.in.rank - 1];
  const int64_t chunk = (P.V + P.ctas - 1) / P.ctas;
  const int64_t j0 = (int64_t)blockIdx.x * chunk, j1 = min(P.V, j0 + chunk);
  float bv = -INFINITY;
  int64_t bi = -1;
  for (int64_t j = j0 + threadIdx.x; j < j1; j += AM_THREADS) am_take(am_load(base, off + j * s_last_dim, P.in.dt), j, bv, bi);
  am_warp(bv, bi);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_v[warp] = bv;
    s_i[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bv = lane < AM_THREADS / 32 ? s_v[lane] : -INFINITY;
    bi = lane < AM_THREADS / 32 ? s_i[lane] : -1;
    am_warp(bv, bi);
  }
  int32_t* out = (int32_t*)dres(P.out, argtab);
  if (P.ctas == 1) {
    if (threadIdx.x == 0) out[row] = (int32_t)(bi < 0 ? 0 : bi);
    return;
  }
  float* pv = (float*)dres(P.part, argtab);
  int64_t* pi = (int64_t*)(pv + P.rows * P.ctas + (P.rows * P.ctas & 1));  // 8-byte aligned after the values
  if (threadIdx.x == 0) {
    pv[row * P.ctas + blockIdx.x] = bv;
    pi[row * P.ctas + blockIdx.x] = bi;
    unsigned* ctr = (unsigned*)dres(P.counters, argtab) + row;
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
    s_last = old == (unsigned)(P.ctas - 1);
  }
  __syncthreads();
  if (!s_last) return;
  // the row's last CTA: every CTA's pair (the acquire above orders these reads)
  bv = -INFINITY;
  bi = -1;
  for (int c = threadIdx.x; c < P.ctas; c += AM_THREADS) am_take(__ldcg(pv + row * P.ctas + c), __ldcg(pi + row * P.ctas + c), bv, bi);
  am_warp(bv, bi);
  __syncthreads();
  if (lane == 0) {
    s_v[warp] = bv;
    s_i[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < AM_THREADS / 32; ++w) am_take(s_v[w], s_i[w], bv, bi);
    out[row] = (int32_t)(bi < 0 ? 0 : bi);
    *((unsigned*)dres(P.counters, argtab) + row) = 0u;  // ready for the next launch
  }
}

}  // namespace

int64_t argmax_part_bytes(const ArgmaxParams& p) {
  const int64_t n = p.rows * p.ctas;
  return (n + (n & 1)) * 4 + n * 8;
}

void launch_argmax(const ArgmaxParams& p, const uint64_t* argtab, cudaStream_t s) {
  launch_k(argmax_kernel, dim3((unsigned)p.ctas, (unsigned)p.rows), dim3(AM_THREADS), 0, s, 1, p, argtab);
}

void verify_argmax(const ArgmaxParams& p, const RegionFn& region) {
  if (p.in.rank < 1 || p.in.rank > CLJXLA_MAXR || p.ctas < 1 || p.ctas > 1024 || p.rows < 1 || p.rows > 65535 ||
      p.V != p.in.shape[p.in.rank - 1])
    fail(E_INTERNAL, "argmax: bad sizes");
  int64_t hi = 0, rows = 1;
  for (int d = 0; d < p.in.rank; ++d) {
    if (p.in.stride[d] < 0) fail(E_INTERNAL, "argmax: negative stride");
    hi += (p.in.shape[d] - 1) * p.in.stride[d];
    if (d + 1 < p.in.rank) rows *= p.in.shape[d];
  }
  if (rows != p.rows) fail(E_INTERNAL, "argmax: row count");
  region(p.in.p, (hi + 1) * (int64_t)dt_size((DT)p.in.dt), "logits");
  region(p.out, p.rows * 4, "token ids");
  if (p.ctas > 1) {
    region(p.part, argmax_part_bytes(p), "partial maxima");
    region(p.counters, p.rows * 4, "arrival counters");
  }
}

}  // namespace cljxla
