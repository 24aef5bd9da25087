// Decode GEMV: y[m, n] = sum_k x[m, k] * W[n, k] for small M (decode batch).
//
// The weight matrices are the only large operands and are read exactly once,
// so the kernel is HBM-bound: every lane streams 16-byte vectors of W with
// no-allocate loads (four independent vectors in flight per lane), x stays in
// L1, accumulation is f32, and each output is rounded once to the result type.
// Rows are split across 1-8 warps (split-K inside the block) so that even
// small projections put enough bytes in flight to cover HBM latency on all
// 148 SMs.  Layout: W row-major [N, K] (the transposed-weight operand of
// clj-xla's Gemma linear layers, gemma.clj:8-23, folded into the kernel).
//
// One launch covers every projection of the same input (q / k / v, gate /
// up): their rows are concatenated into one index space of segments.  The
// kernel is launched as a programmatic dependent of the kernel before it and
// asks L2 for its weight rows before waiting for that kernel, so the weight
// stream starts while the previous (small) kernel is still running.
#include <cuda_bf16.h>

#include "fast_kernels.h"

namespace cljxla {
namespace {

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// 8 consecutive x values (bf16 or f32) as f32
template <typename XT>
__device__ __forceinline__ void load_x8(const XT* x, float* o);
template <>
__device__ __forceinline__ void load_x8<uint16_t>(const uint16_t* x, float* o) {
  uint4 v = *(const uint4*)x;
  o[0] = bf_lo(v.x); o[1] = bf_hi(v.x); o[2] = bf_lo(v.y); o[3] = bf_hi(v.y);
  o[4] = bf_lo(v.z); o[5] = bf_hi(v.z); o[6] = bf_lo(v.w); o[7] = bf_hi(v.w);
}
template <>
__device__ __forceinline__ void load_x8<float>(const float* x, float* o) {
  float4 a = *(const float4*)x, b = *(const float4*)(x + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

__device__ __forceinline__ float dot8(const uint4& w, const float* x) {
  float s = bf_lo(w.x) * x[0];
  s = fmaf(bf_hi(w.x), x[1], s);
  s = fmaf(bf_lo(w.y), x[2], s);
  s = fmaf(bf_hi(w.y), x[3], s);
  s = fmaf(bf_lo(w.z), x[4], s);
  s = fmaf(bf_hi(w.z), x[5], s);
  s = fmaf(bf_lo(w.w), x[6], s);
  s = fmaf(bf_hi(w.w), x[7], s);
  return s;
}

__device__ __forceinline__ void store_out(char* y, int64_t i, int dt, float v) {
  if (dt == KDT_F32) ((float*)y)[i] = v;
  else ((__nv_bfloat16*)y)[i] = __float2bfloat16_rn(v);
}

template <int MT, typename XT>
__global__ void __launch_bounds__(256) gemv_nt_bf16(const __grid_constant__ GemvParams P,
                                                   const uint64_t* __restrict__ argtab) {
  __shared__ float red[8][MT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpr = P.warps_per_row;
  const int rows_per_block = 8 / wpr;
  const int part = warp % wpr;
  const int64_t kper = P.K / wpr;  // multiple of 8 (checked on the host)
  const int64_t k0 = part * kper, k1 = (part == wpr - 1) ? P.K : k0 + kper;
  const int64_t stride = (int64_t)gridDim.x * rows_per_block;
  // weights do not depend on the previous kernel: start this warp's rows towards L2 now
  for (int64_t row = (int64_t)blockIdx.x * rows_per_block + warp / wpr; row < P.N; row += stride) {
    int sg = 0;
    while (sg < P.nseg - 1 && row >= P.seg_end[sg]) ++sg;
    const uint16_t* wrow = (const uint16_t*)dres(P.w[sg], argtab) + (row - (sg ? P.seg_end[sg - 1] : 0)) * P.K;
    for (int64_t k = k0 + lane * 64; k < k1; k += 32 * 64) prefetch_l2(wrow + k);
  }
  pdl_enter();
  const XT* X = (const XT*)dres(P.x, argtab);
  // every warp of the block runs the same number of rounds (block-uniform bound)
  for (int64_t base = (int64_t)blockIdx.x * rows_per_block; base < P.N; base += stride) {
    const int64_t row = base + warp / wpr;
    const bool active = row < P.N;
    int sg = 0;
    while (sg < P.nseg - 1 && row >= P.seg_end[sg]) ++sg;
    const int64_t lrow = row - (sg ? P.seg_end[sg - 1] : 0);
    const uint16_t* wrow = (const uint16_t*)dres(P.w[sg], argtab) + lrow * P.K;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    if (active) {
      int64_t k = k0 + lane * 8;
      // main loop: 4 independent 16-byte weight vectors in flight per lane
      for (; k + 3 * 256 < k1; k += 4 * 256) {
        uint4 w0 = ld_stream(wrow + k), w1 = ld_stream(wrow + k + 256), w2 = ld_stream(wrow + k + 512),
              w3 = ld_stream(wrow + k + 768);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float xv[8];
          const XT* xr = X + m * P.x_sm;
          load_x8<XT>(xr + k, xv);
          float s = dot8(w0, xv);
          load_x8<XT>(xr + k + 256, xv);
          s += dot8(w1, xv);
          load_x8<XT>(xr + k + 512, xv);
          s += dot8(w2, xv);
          load_x8<XT>(xr + k + 768, xv);
          s += dot8(w3, xv);
          acc[m] += s;
        }
      }
      for (; k < k1; k += 256) {
        uint4 w0 = ld_stream(wrow + k);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float xv[8];
          load_x8<XT>(X + m * P.x_sm + k, xv);
          acc[m] += dot8(w0, xv);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], s);
    if (wpr > 1) {
      if (lane == 0)
#pragma unroll
        for (int m = 0; m < MT; ++m) red[warp][m] = acc[m];
      __syncthreads();
      if (part == 0 && lane == 0 && active) {
        for (int q = 1; q < wpr; ++q)
#pragma unroll
          for (int m = 0; m < MT; ++m) acc[m] += red[warp + q][m];
      }
      __syncthreads();  // red is rewritten next round
    }
    if (active && part == 0 && lane == 0) {
      char* Y = dres(P.y[sg], argtab);
      const int64_t nseg_rows = P.seg_end[sg] - (sg ? P.seg_end[sg - 1] : 0);
#pragma unroll
      for (int m = 0; m < MT; ++m) store_out(Y, m * nseg_rows + lrow, P.y_dt[sg], acc[m]);
    }
  }
  // this CTA's share of the next GEMV's weights: one bulk L2 prefetch per segment
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.npf; ++i) {
      const int64_t per = ((P.pf_bytes[i] / gridDim.x) + 15) & ~(int64_t)15;
      const int64_t lo = per * blockIdx.x;
      int64_t n = P.pf_bytes[i] - lo;
      if (n > per) n = per;
      if (n <= 0) continue;
      const char* src = dres(P.pf[i], argtab) + lo;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"((uint32_t)n) : "memory");
    }
  }
}

// Launch shape: the grid is at most one wave of resident blocks, each block
// striding over row groups; the K split per row (1-8 warps) is the one with
// the least quantised work per warp, iterations x (K / split + 128).
struct GemvShape {
  int wpr;
  unsigned grid;
};

GemvShape gemv_shape(int64_t N, int64_t K, int resident_blocks) {
  GemvShape best{1, 1};
  double best_cost = 1e300;
  for (int wpr = 1; wpr <= 8; wpr *= 2) {
    if (wpr > 1 && ((K / wpr) % 8 != 0 || K / wpr < 256)) break;
    const int64_t rpb = 8 / wpr;
    const int64_t groups = (N + rpb - 1) / rpb;
    const int64_t grid = std::min<int64_t>(groups, resident_blocks);
    const int64_t iters = (groups + grid - 1) / grid;
    const double cost = (double)iters * ((double)K / wpr + 128.0);
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = GemvShape{wpr, (unsigned)grid};
    }
  }
  return best;
}

template <int MT, typename XT>
void launch_nt_t(GemvParams p, const uint64_t* argtab, cudaStream_t s) {
  static int per_sm = 0;  // occupancy is a property of the kernel on sm_100a, the same on every B200
  if (!per_sm) {
    int v = 1;
    CUDA_OK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, gemv_nt_bf16<MT, XT>, 256, 0));
    per_sm = std::max(1, v);
  }
  const int resident = device_sm_count() * per_sm;
  GemvShape sh = gemv_shape(p.N, p.K, resident);
  p.warps_per_row = sh.wpr;
  launch_k(gemv_nt_bf16<MT, XT>, dim3(sh.grid), dim3(256), 0, s, 1, p, argtab);
}

template <int MT>
void launch_nt(const GemvParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.x_dt == KDT_F32) launch_nt_t<MT, float>(p, argtab, s);
  else launch_nt_t<MT, uint16_t>(p, argtab, s);
}

int choose_warps_per_row(int64_t N, int64_t K) {
  // enough warps in flight: split K across up to 8 warps per row
  int wpr = 1;
  while (wpr < 8 && N * wpr < 148 * 48 && (K / (wpr * 2)) % 8 == 0 && K / (wpr * 2) >= 256) wpr *= 2;
  return wpr;
}

bool gemv_shape_ok(const GemmParams& g) {
  // decode shapes only: one batch, few rows, bf16 weights laid out [N, K]
  // CLJXLA_B200_GEMV_MAX_ROWS (default 8): more rows take the tensor-core GEMM
  static const int max_rows = [] {
    const char* e = getenv("CLJXLA_B200_GEMV_MAX_ROWS");
    return e && atoi(e) >= 1 ? std::min(8, atoi(e)) : 8;
  }();
  if (g.batch != 1 || g.M < 1 || g.M > max_rows || g.b_dt != KDT_BF16) return false;
  if (!(g.a_dt == KDT_BF16 || g.a_dt == KDT_F32) || !(g.c_dt == KDT_BF16 || g.c_dt == KDT_F32)) return false;
  if (g.b_sk != 1 || g.b_sn != g.K || g.a_sk != 1) return false;
  if (g.K % 8 != 0 || g.K < 256) return false;
  if ((g.b.off % 16) != 0 || (g.a.off % 16) != 0) return false;
  if (g.M > 1 && (g.a_sm % 8) != 0) return false;
  if (g.M == 5 || g.M == 6 || g.M == 7) return false;  // keep the M=8 path exact-sized
  return true;
}

}  // namespace

void launch_gemv(const GemvParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.N == 0) return;
  switch (p.M) {
    case 1: launch_nt<1>(p, argtab, s); break;
    case 2: launch_nt<2>(p, argtab, s); break;
    case 3: launch_nt<3>(p, argtab, s); break;
    case 4: launch_nt<4>(p, argtab, s); break;
    case 5: case 6: case 7: case 8: launch_nt<8>(p, argtab, s); break;
    default: fail(E_INTERNAL, "gemv: unsupported M");
  }
}

bool make_gemv(const GemmParams& g, Launch& out) {
  if (!gemv_shape_ok(g)) return false;
  GemvParams p{};
  p.x = g.a;
  p.w[0] = g.b;
  p.y[0] = g.c;
  p.y_dt[0] = g.c_dt;
  p.seg_end[0] = g.N;
  p.nseg = 1;
  p.x_dt = g.a_dt;
  p.w_dt = g.b_dt;
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.x_sm = g.a_sm;
  p.warps_per_row = choose_warps_per_row(p.N, p.K);
  out.kind = K_GEMV;
  out.blob.resize(sizeof(p));
  memcpy(out.blob.data(), &p, sizeof(p));
  return true;
}

bool gemv_add_segment(Launch& l, const GemmParams& g) {
  if (l.kind != K_GEMV || !gemv_shape_ok(g)) return false;
  GemvParams p;
  memcpy(&p, l.blob.data(), sizeof(p));
  if (p.nseg >= GEMV_MAXSEG || g.M != p.M || g.K != p.K || g.a_dt != p.x_dt || g.a_sm != p.x_sm ||
      g.a.slot != p.x.slot || g.a.off != p.x.off)
    return false;
  p.w[p.nseg] = g.b;
  p.y[p.nseg] = g.c;
  p.y_dt[p.nseg] = g.c_dt;
  p.N += g.N;
  p.seg_end[p.nseg] = p.N;
  p.nseg++;
  p.warps_per_row = choose_warps_per_row(p.N, p.K);
  memcpy(l.blob.data(), &p, sizeof(p));
  return true;
}

void link_gemv_prefetch(Plan& plan) {
  // off by default: on Gemma-3-4B decode 8 MB changed nothing and 24 / 48 MB
  // cost 1-3 % (the prefetch competes with the tail of the running GEMV);
  // CLJXLA_B200_GEMV_PREFETCH_MB sets a budget
  int64_t kMaxPrefetch = 0;
  if (const char* e = getenv("CLJXLA_B200_GEMV_PREFETCH_MB")) kMaxPrefetch = atoll(e) << 20;
  GemvParams* prev = nullptr;
  Launch* prev_l = nullptr;
  for (Launch& l : plan.launches) {
    if (l.kind != K_GEMV) continue;
    GemvParams cur;
    memcpy(&cur, l.blob.data(), sizeof(cur));
    if (prev) {
      GemvParams& p = *prev;
      p.npf = 0;
      int64_t budget = kMaxPrefetch;
      for (int i = 0; i < cur.nseg && budget > 0; ++i) {
        const int64_t n = cur.seg_end[i] - (i ? cur.seg_end[i - 1] : 0);
        int64_t bytes = std::min<int64_t>(n * cur.K * 2, budget) & ~(int64_t)15;
        if (bytes <= 0) break;
        p.pf[p.npf] = cur.w[i];
        p.pf_bytes[p.npf] = bytes;
        p.npf++;
        budget -= bytes;
      }
      memcpy(prev_l->blob.data(), prev, sizeof(GemvParams));
    }
    prev_l = &l;
    prev = (GemvParams*)l.blob.data();
  }
}

void link_attention_hints(Plan& plan) {
  // the HBM idles while a decode attention runs (its K / V come from L2,
  // prefetched during the kernel before it): the attention asks L2 for the
  // weights of the GEMVs after it, in launch order, up to CLJXLA_B200_L2_HINT_MB
  // (off by default: the prefetch slowed the step down at every budget tried)
  int64_t budget_all = 0;  // measured: 24 / 64 / 112 / 160 MB cost 1 / 2 / 4 / 10 % on Gemma-3-4B decode
  if (const char* e = getenv("CLJXLA_B200_L2_HINT_MB")) budget_all = atoll(e) << 20;
  const int n = (int)plan.launches.size();
  for (int i = 0; i < n; ++i) {
    Launch& l = plan.launches[i];
    if (l.kind != K_ATTN_DECODE) continue;
    AttnParams& a = *(AttnParams*)l.blob.data();
    a.nhint = 0;
    if (a.use_tc != 3 || budget_all <= 0) continue;
    int64_t budget = budget_all;
    for (int j = i + 1; j < n && budget > 0 && a.nhint < ATTN_MAX_HINTS; ++j) {
      const Launch& g = plan.launches[j];
      if (g.kind == K_ATTN_DECODE) break;  // the next layer's attention prefetches its own
      if (g.kind != K_GEMV) continue;
      const GemvParams& gp = *(const GemvParams*)g.blob.data();
      if (gp.w_dt != KDT_BF16 && gp.w_dt != KDT_F32) continue;
      const int64_t es = gp.w_dt == KDT_F32 ? 4 : 2;
      for (int s = 0; s < gp.nseg && budget > 0 && a.nhint < ATTN_MAX_HINTS; ++s) {
        if (gp.w[s].off % 16) continue;
        const int64_t rows = gp.seg_end[s] - (s ? gp.seg_end[s - 1] : 0);
        const int64_t bytes = std::min<int64_t>(rows * gp.K * es, budget) & ~(int64_t)15;
        if (bytes <= 0) break;
        a.hint[a.nhint] = gp.w[s];
        a.hint_bytes[a.nhint] = bytes;
        a.nhint++;
        budget -= bytes;
      }
    }
  }
}

void verify_gemv(const Plan& plan, const Launch& l, const RegionFn& region) {
  (void)plan;
  const GemvParams& p = *(const GemvParams*)l.blob.data();
  if (p.npf < 0 || p.npf > GEMV_MAXSEG) fail(E_INTERNAL, "gemv: bad prefetch list");
  for (int i = 0; i < p.npf; ++i) {
    if (p.pf_bytes[i] % 16 || p.pf[i].off % 16) fail(E_INTERNAL, "gemv: unaligned prefetch");
    region(p.pf[i], p.pf_bytes[i], "prefetched weights");
  }
  if (p.nseg < 1 || p.nseg > GEMV_MAXSEG || p.seg_end[p.nseg - 1] != p.N) fail(E_INTERNAL, "gemv: bad segments");
  if (p.has_status) region(p.status, 4, "status word");
  int64_t xs = dt_size((DT)p.x_dt);
  region(p.x, ((p.M - 1) * p.x_sm + p.K) * xs, "x");
  for (int i = 0; i < p.nseg; ++i) {
    const int64_t n = p.seg_end[i] - (i ? p.seg_end[i - 1] : 0);
    if (n <= 0) fail(E_INTERNAL, "gemv: empty segment");
    region(p.w[i], n * p.K * 2, "weights");
    region(p.y[i], p.M * n * (int64_t)dt_size((DT)p.y_dt[i]), "y");
  }
}

}  // namespace cljxla
