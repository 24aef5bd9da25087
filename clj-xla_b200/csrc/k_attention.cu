// Fused grouped-query attention over a KV cache (flash-decoding).
//
// Replaces the printed attention block of attention.clj:343-365
//   scores = dot_general(q, reshape(broadcast_in_dim(K)))      (GQA broadcast)
//   s      = <scale / softcap chain>(scores)                    (printed as bf16 ops)
//   m      = s + mask ; p = exp(m - max m) / sum exp(...)       (f32 softmax)
//   out    = dot_general(p, reshape(broadcast_in_dim(V)))
// with one kernel that reads each K/V row once per KV head (all query heads of
// the group share it), keeps the softmax online in registers, and never
// materialises the broadcast K/V, the score matrix or the probabilities.
//
// Grid: (position splits, query tiles, batch * kv heads); 4 warps per CTA,
// each warp walks positions of the CTA's chunk; per position a lane owns
// hd/32 consecutive elements of the K and V rows.  Partial (max, sum, acc)
// triples are merged across warps in shared memory and, when the positions
// are split across CTAs, across CTAs by attn_combine.
//
// Positions whose additive mask is at or below `mask_skip` for every query
// row of the CTA are skipped without loading K/V.  This is exact for the
// causal / sliding-window masks the reference prints (-10000,
// attention.clj:208,224): such a position's softmax weight
// exp(s - 10000 - max) underflows to exactly 0 in f32 whenever the unmasked
// scores lie within ~4900 of each other.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fast_kernels.h"

namespace cljxla {
namespace {

__device__ __forceinline__ float rnd_dt(float v, int dt) {
  if (dt == KDT_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == KDT_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ float ld_any(const char* base, int64_t i, int dt) {
  if (dt == KDT_F32) return ((const float*)base)[i];
  if (dt == KDT_BF16) return __uint_as_float((uint32_t)((const uint16_t*)base)[i] << 16);
  return __half2float(((const __half*)base)[i]);
}

// HPL consecutive K/V elements of one row as f32
template <typename KT, int HPL>
__device__ __forceinline__ void load_row(const KT* p, float* o);

template <>
__device__ __forceinline__ void load_row<uint16_t, 8>(const uint16_t* p, float* o) {
  uint4 v = *(const uint4*)p;
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) { o[2 * i] = __uint_as_float(w[i] << 16); o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u); }
}
template <>
__device__ __forceinline__ void load_row<uint16_t, 4>(const uint16_t* p, float* o) {
  uint2 v = *(const uint2*)p;
  o[0] = __uint_as_float(v.x << 16); o[1] = __uint_as_float(v.x & 0xffff0000u);
  o[2] = __uint_as_float(v.y << 16); o[3] = __uint_as_float(v.y & 0xffff0000u);
}
template <>
__device__ __forceinline__ void load_row<uint16_t, 2>(const uint16_t* p, float* o) {
  uint32_t v = *(const uint32_t*)p;
  o[0] = __uint_as_float(v << 16); o[1] = __uint_as_float(v & 0xffff0000u);
}
template <>
__device__ __forceinline__ void load_row<uint16_t, 1>(const uint16_t* p, float* o) {
  o[0] = __uint_as_float((uint32_t)p[0] << 16);
}
template <int HPL>
__device__ __forceinline__ void load_row_f32(const float* p, float* o) {
#pragma unroll
  for (int i = 0; i < HPL; ++i) o[i] = p[i];
}
template <>
__device__ __forceinline__ void load_row<float, 1>(const float* p, float* o) { load_row_f32<1>(p, o); }
template <>
__device__ __forceinline__ void load_row<float, 2>(const float* p, float* o) {
  float2 v = *(const float2*)p;
  o[0] = v.x; o[1] = v.y;
}
template <>
__device__ __forceinline__ void load_row<float, 4>(const float* p, float* o) {
  float4 v = *(const float4*)p;
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
template <>
__device__ __forceinline__ void load_row<float, 8>(const float* p, float* o) {
  float4 a = *(const float4*)p, b = *(const float4*)(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

// the printed scale / softcap chain applied to one score (register 0 holds it)
__device__ __noinline__ float run_chain(const AttnParams& P, float s) {
  float R[16];
  R[0] = s;
  for (int pc = 0; pc < P.nchain; ++pc) {
    const EwInstr& I = P.chain[pc];
    float a = R[I.a], b = R[I.b], z;
    switch (I.op) {
      case EW_IMM: z = I.fimm; break;
      case EW_ADD: z = a + b; break;
      case EW_SUB: z = a - b; break;
      case EW_MUL: z = a * b; break;
      case EW_DIV: z = a / b; break;
      case EW_MAX: z = fmaxf(a, b); break;
      case EW_MIN: z = fminf(a, b); break;
      case EW_TANH: z = tanhf(a); break;
      case EW_NEG: z = -a; break;
      case EW_CONVERT: z = a; break;
      default: z = a; break;
    }
    R[I.dst] = rnd_dt(z, I.dt);
  }
  return R[P.chain_out];
}

// the chain in its closed form where the planner found one
__device__ __forceinline__ float apply_chain(const AttnParams& P, float s) {
  if (P.chain_kind == 1) return rnd_dt(s * P.chain_c, P.chain_dt);
  if (P.chain_kind == 2) return s;
  return run_chain(P, s);
}

constexpr int NW = 4;

// merged (max, sum, context) of one output row over the position splits, in
// split order (the same arithmetic as attn_combine_kernel)
__device__ __forceinline__ float merge_splits(const float* part, int64_t rows_total, int64_t row, int HD, int d,
                                              int splits) {
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, __ldcg(part + ((int64_t)s * rows_total + row) * (HD + 2)));
  float L = 0.f, A = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float* pp = part + ((int64_t)s * rows_total + row) * (HD + 2);
      const float pm = __ldcg(pp);
      if (pm == -INFINITY) continue;
      float sc = expf(pm - M);
      L += __ldcg(pp + 1) * sc;
      A += __ldcg(pp + 2 + d) * sc;
    }
  }
  return L > 0.f ? A / L : 0.f;
}

// With per-launch arrival counters, the last split CTA of a (batch*kv head,
// query tile) merges everyone's partials (threadfence-ordered, no waiting).
// One warp per query vector turns the splits' (max, sum) pairs into scale
// factors in shared memory; then every thread forms two output columns from
// all splits with independent 8-byte loads.
__device__ void merge_if_last(const AttnParams& P, const uint64_t* __restrict__ argtab, int b, int kh, int i0,
                              int nqv) {
  if (P.splits == 1 || !P.use_counters) return;
  __shared__ int s_last;
  __shared__ float s_sc[ATTN_MERGE_MAX_SPLITS][8];
  __shared__ float s_pl[ATTN_MERGE_MAX_SPLITS][8];
  __shared__ float s_l[8];
  // the barrier orders every thread's partial stores before thread 0's release;
  // the acquire of the last arrival orders its reads after everyone's stores
  __syncthreads();
  unsigned* ctr = (unsigned*)dres(P.counters, argtab) + ((int64_t)blockIdx.z * gridDim.y + blockIdx.y);
  if (threadIdx.x == 0) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
    s_last = old == (unsigned)(P.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  const int64_t rows_total = (int64_t)P.B * P.nq * P.Sq;
  const float* part = (const float*)dres(P.part, argtab);
  char* ob = dres(P.out, argtab);
  const int HD = P.hd, S = P.splits;
  auto row_of = [&](int r) {
    const int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
    return ((int64_t)b * P.nq + h) * P.Sq + qi;
  };
  // every split's (max, sum) of every row at once, then the scale factors
  for (int e = threadIdx.x; e < S * nqv; e += blockDim.x) {
    const int sp = e / nqv, r = e % nqv;
    const float* pp = part + ((int64_t)sp * rows_total + row_of(r)) * (HD + 2);
    s_sc[sp][r] = __ldcg(pp);
    s_pl[sp][r] = __ldcg(pp + 1);
  }
  __syncthreads();
  // one warp per row: the splits' maximum, their scale factors and the sum
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < nqv; r += nw) {
    float m = -INFINITY;
    for (int sp = lane; sp < S; sp += 32) m = fmaxf(m, s_sc[sp][r]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int sp = lane; sp < S; sp += 32) {
      const float pm = s_sc[sp][r];
      const float sc = (m == -INFINITY || pm == -INFINITY) ? 0.f : expf(pm - m);
      s_sc[sp][r] = sc;
      l += sc == 0.f ? 0.f : s_pl[sp][r] * sc;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) s_l[r] = l;
  }
  __syncthreads();
  const int half = HD / 2;
  for (int e = threadIdx.x; e < nqv * half; e += blockDim.x) {
    const int r = e / half, d = 2 * (e % half);
    const int64_t row = row_of(r);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < S; ++sp) {
      const float2 v = __ldcg((const float2*)(part + ((int64_t)sp * rows_total + row) * (HD + 2) + 2 + d));
      const float sc = s_sc[sp][r];
      a0 += v.x * sc;
      a1 += v.y * sc;
    }
    const float l = s_l[r];
    const float o0 = l > 0.f ? a0 / l : 0.f, o1 = l > 0.f ? a1 / l : 0.f;
    if (P.out_dt == KDT_F32) {
      ((float*)ob)[row * HD + d] = o0;
      ((float*)ob)[row * HD + d + 1] = o1;
    } else {
      ((__nv_bfloat16*)ob)[row * HD + d] = __float2bfloat16_rn(o0);
      ((__nv_bfloat16*)ob)[row * HD + d + 1] = __float2bfloat16_rn(o1);
    }
  }
  if (threadIdx.x == 0) *ctr = 0u;  // ready for the next launch
}


// The additive mask of query row offset `moff` at position j.  mask_mode 0
// reads it through the mask view; mask_mode 1 computes the causal /
// sliding-window form the planner proved the printed mask to be, where the
// view's strides {0, 0, 1, 0} make `moff` the query index and qpos0 is the
// position of query 0 (mask_qpos0: the graph's position parameter plus the
// form's offset).  The position parameter is never written by a plan kernel,
// so it may be read before a kernel's dependency wait.
__device__ __forceinline__ int mask_qpos0(const AttnParams& P, const uint64_t* __restrict__ argtab) {
  if (!P.mask_mode) return 0;
  return P.mask_off + (P.has_mask_pos ? *(const int*)dres(P.mask_pos, argtab) : 0);
}
__device__ __forceinline__ float mask_at(const AttnParams& P, const char* mb, int64_t moff, int64_t j, int qpos0) {
  if (P.mask_mode) {
    const int d = (int)j - (qpos0 + (int)moff);
    return (d > P.mask_gt || d < P.mask_lt) ? P.mask_mv : P.mask_z;
  }
  return ld_any(mb, moff + j * P.mask.stride[3], P.mask.dt);
}
template <typename KT, int HPL, int NQV>
__global__ void __launch_bounds__(NW * 32) attn_kernel(const __grid_constant__ AttnParams P,
                                                      const uint64_t* __restrict__ argtab) {
  pdl_enter();
  constexpr int HD = HPL * 32;
  __shared__ float qs[NQV][HD];
  __shared__ float wm[NW][NQV], wl[NW][NQV];
  __shared__ float wacc[NW][NQV][HD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bk = blockIdx.z;
  const int b = bk / P.nkv, kh = bk % P.nkv;
  const int i0 = blockIdx.y * P.qtile;
  const int nrows = min(P.qtile, P.Sq - i0);
  const int nqv = nrows * P.group;  // active query vectors: r = qi * group + gi
  const int split = blockIdx.x;
  const int64_t chunk = (P.T + P.splits - 1) / P.splits;
  const int64_t t0 = split * chunk, t1 = min((int64_t)P.T, t0 + chunk);
  const char* qb = dres(P.q.p, argtab);
  const KT* kb = (const KT*)dres(P.k.p, argtab);
  const KT* vb = (const KT*)dres(P.v.p, argtab);
  const char* mb = dres(P.mask.p, argtab);
  const int qp0 = mask_qpos0(P, argtab);

  // query vectors of this CTA -> shared (f32)
  for (int e = threadIdx.x; e < NQV * HD; e += NW * 32) {
    int r = e / HD, d = e % HD;
    float val = 0.f;
    if (r < nqv) {
      int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
      val = ld_any(qb, b * P.q.stride[0] + h * P.q.stride[1] + qi * P.q.stride[2] + d * P.q.stride[3], P.q.dt);
    }
    qs[r][d] = val;
  }
  __syncthreads();

  float m[NQV], l[NQV], acc[NQV][HPL];
#pragma unroll
  for (int r = 0; r < NQV; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < HPL; ++e) acc[r][e] = 0.f;
  }
  const KT* kbase = kb + b * P.k.stride[0] + kh * P.k.stride[1];
  const KT* vbase = vb + b * P.v.stride[0] + kh * P.v.stride[1] + lane * HPL;
  int64_t mrow[NQV];
#pragma unroll
  for (int r = 0; r < NQV; ++r) {
    const int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
    mrow[r] = r < nqv ? b * P.mask.stride[0] + h * P.mask.stride[1] + qi * P.mask.stride[2] : 0;
  }
  // Rounds of 32 positions per warp: each lane owns one position for the scores
  // (the whole q.k dot product of its own K row, no shuffles), the round's
  // softmax statistics are warp reductions, and the P.V product walks the
  // round's unmasked positions with each lane owning hd/32 output elements.
  for (int64_t j0 = t0 + (int64_t)warp * 32; j0 < t1; j0 += NW * 32) {
    const int64_t j = j0 + lane;
    float mk[NQV];
    bool any = false;
#pragma unroll
    for (int r = 0; r < NQV; ++r) {
      mk[r] = -INFINITY;
      if (r < nqv && j < t1) {
        mk[r] = mask_at(P, mb, mrow[r], j, qp0);
        any |= mk[r] > P.mask_skip;
      }
    }
    const unsigned valid = __ballot_sync(0xffffffffu, any);
    if (!valid) continue;
    float s[NQV];
#pragma unroll
    for (int r = 0; r < NQV; ++r) s[r] = 0.f;
    if (any) {
      const KT* krow = kbase + j * P.k.stride[2];
#pragma unroll 4
      for (int c = 0; c < HD; c += HPL) {
        float kr[HPL];
        load_row<KT, HPL>(krow + c, kr);
#pragma unroll
        for (int r = 0; r < NQV; ++r)
#pragma unroll
          for (int e = 0; e < HPL; ++e) s[r] = fmaf(qs[r][c + e], kr[e], s[r]);
      }
    }
    float p[NQV];
#pragma unroll
    for (int r = 0; r < NQV; ++r) {
      p[r] = 0.f;
      if (r >= nqv) continue;  // uniform across the warp
      float mv = -INFINITY;
      if (any) mv = rnd_dt(apply_chain(P, rnd_dt(s[r], P.dt_d1)) + mk[r], P.dt_m);
      float rm = mv;
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1) rm = fmaxf(rm, __shfl_xor_sync(0xffffffffu, rm, sh));
      const float mnew = fmaxf(m[r], rm);
      if (mnew == -INFINITY) continue;  // uniform
      if (any) p[r] = rnd_dt(expf(rnd_dt(mv - mnew, P.dt_sub)), P.dt_exp);
      float ps = p[r];
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, sh);
      const float sc = m[r] == -INFINITY ? 0.f : expf(m[r] - mnew);
      l[r] = l[r] * sc + ps;
#pragma unroll
      for (int e = 0; e < HPL; ++e) acc[r][e] *= sc;
      m[r] = mnew;
    }
    // P.V: four unmasked positions per step so their V rows load together
    unsigned bits = valid;
    while (bits) {
      int src[4];
      int cnt = 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        src[u] = bits ? __ffs(bits) - 1 : -1;
        if (bits) { bits &= bits - 1; ++cnt; }
      }
      float vr[4][HPL];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (src[u] >= 0) load_row<KT, HPL>(vbase + (j0 + src[u]) * P.v.stride[2], vr[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (src[u] < 0) break;  // uniform
#pragma unroll
        for (int r = 0; r < NQV; ++r) {
          const float pj = __shfl_sync(0xffffffffu, p[r], src[u]);
#pragma unroll
          for (int e = 0; e < HPL; ++e) acc[r][e] = fmaf(pj, vr[u][e], acc[r][e]);
        }
      }
      (void)cnt;
    }
  }
  // merge warps
#pragma unroll
  for (int r = 0; r < NQV; ++r) {
    if (lane == 0) { wm[warp][r] = m[r]; wl[warp][r] = l[r]; }
#pragma unroll
    for (int e = 0; e < HPL; ++e) wacc[warp][r][lane * HPL + e] = acc[r][e];
  }
  __syncthreads();
  const int64_t rows_total = (int64_t)P.B * P.nq * P.Sq;
  for (int e = threadIdx.x; e < nqv * HD; e += NW * 32) {
    int r = e / HD, d = e % HD;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][r]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < NW; ++w) {
        float sc = wm[w][r] == -INFINITY ? 0.f : expf(wm[w][r] - M);
        L += wl[w][r] * sc;
        A += wacc[w][r][d] * sc;
      }
    }
    int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
    int64_t row = ((int64_t)b * P.nq + h) * P.Sq + qi;
    if (P.splits == 1) {
      float o = L > 0.f ? A / L : 0.f;
      char* ob = dres(P.out, argtab);
      if (P.out_dt == KDT_F32) ((float*)ob)[row * HD + d] = o;
      else ((__nv_bfloat16*)ob)[row * HD + d] = __float2bfloat16_rn(o);
    } else {
      float* part = (float*)dres(P.part, argtab) + ((int64_t)split * rows_total + row) * (HD + 2);
      part[2 + d] = A;
      if (d == 0) { part[0] = M; part[1] = L; }
    }
  }
  merge_if_last(P, argtab, b, kh, i0, nqv);
}

// ---------------------------------------------------------------------------
// bf16 K/V with 16-byte aligned rows: each sub-chunk of CH positions is first
// staged in shared memory with cp.async (only the rows between the first and
// last unmasked position), so every K/V byte the CTA needs is in flight at
// once instead of one row per dependent load.  Rows are padded by 16 bytes so
// that lanes reading different rows at the same column hit different banks.
constexpr int CH = 128;  // positions per staged sub-chunk (one 32-position round per warp)

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
               : "memory");
}

template <int HPL, int NQV>
__global__ void __launch_bounds__(NW * 32) attn_smem_kernel(const __grid_constant__ AttnParams P,
                                                           const uint64_t* __restrict__ argtab) {
  pdl_enter();
  constexpr int HD = HPL * 32;
  constexpr int ROW = HD + 8;  // padded row, bf16 elements
  extern __shared__ __align__(16) uint16_t kv_smem[];
  uint16_t* Ks = kv_smem;
  uint16_t* Vs = kv_smem + CH * ROW;
  __shared__ float qs[NQV][HD];
  __shared__ float wm[NW][NQV], wl[NW][NQV];
  __shared__ float wacc[NW][NQV][HD];
  __shared__ int s_lo, s_hi;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bk = blockIdx.z;
  const int b = bk / P.nkv, kh = bk % P.nkv;
  const int i0 = blockIdx.y * P.qtile;
  const int nrows = min(P.qtile, P.Sq - i0);
  const int nqv = nrows * P.group;
  const int split = blockIdx.x;
  const int64_t chunk = (P.T + P.splits - 1) / P.splits;
  const int64_t t0 = split * chunk, t1 = min((int64_t)P.T, t0 + chunk);
  const char* qb = dres(P.q.p, argtab);
  const uint16_t* kbase = (const uint16_t*)dres(P.k.p, argtab) + b * P.k.stride[0] + kh * P.k.stride[1];
  const uint16_t* vbase = (const uint16_t*)dres(P.v.p, argtab) + b * P.v.stride[0] + kh * P.v.stride[1];
  const char* mb = dres(P.mask.p, argtab);
  const int qp0 = mask_qpos0(P, argtab);

  for (int e = threadIdx.x; e < NQV * HD; e += NW * 32) {
    int r = e / HD, d = e % HD;
    float val = 0.f;
    if (r < nqv) {
      int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
      val = ld_any(qb, b * P.q.stride[0] + h * P.q.stride[1] + qi * P.q.stride[2] + d * P.q.stride[3], P.q.dt);
    }
    qs[r][d] = val;
  }
  int64_t mrow[NQV];
#pragma unroll
  for (int r = 0; r < NQV; ++r) {
    const int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
    mrow[r] = r < nqv ? b * P.mask.stride[0] + h * P.mask.stride[1] + qi * P.mask.stride[2] : 0;
  }
  float m[NQV], l[NQV], acc[NQV][HPL];
#pragma unroll
  for (int r = 0; r < NQV; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < HPL; ++e) acc[r][e] = 0.f;
  }
  for (int64_t c0 = t0; c0 < t1; c0 += CH) {
    const int64_t c1 = min(t1, c0 + CH);
    // this thread's position: mask values and whether any query vector sees it
    const int64_t j = c0 + warp * 32 + lane;
    float mk[NQV];
    bool any = false;
#pragma unroll
    for (int r = 0; r < NQV; ++r) {
      mk[r] = -INFINITY;
      if (r < nqv && j < c1) {
        mk[r] = mask_at(P, mb, mrow[r], j, qp0);
        any |= mk[r] > P.mask_skip;
      }
    }
    if (threadIdx.x == 0) { s_lo = CH; s_hi = -1; }
    __syncthreads();  // also orders the previous sub-chunk's reads before the restaging below
    if (any) {
      atomicMin(&s_lo, (int)(j - c0));
      atomicMax(&s_hi, (int)(j - c0));
    }
    __syncthreads();
    const int lo = s_lo, hi = s_hi;
    if (hi < lo) continue;  // the whole sub-chunk is masked
    // stage rows [lo, hi] of K and V
    constexpr int SEGS = HD * 2 / 16;  // 16-byte pieces per row
    const int nseg = (hi - lo + 1) * SEGS;
    for (int q = threadIdx.x; q < nseg; q += NW * 32) {
      const int rr = lo + q / SEGS, sg = q % SEGS;
      cp_async16(Ks + rr * ROW + sg * 8, kbase + (c0 + rr) * P.k.stride[2] + sg * 8);
      cp_async16(Vs + rr * ROW + sg * 8, vbase + (c0 + rr) * P.v.stride[2] + sg * 8);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // scores: lane = position warp*32+lane of the sub-chunk
    const int pl = warp * 32 + lane;
    const unsigned valid = __ballot_sync(0xffffffffu, any);
    if (valid) {
      float s[NQV];
#pragma unroll
      for (int r = 0; r < NQV; ++r) s[r] = 0.f;
      if (any) {
        // two partial sums per row (even / odd 8-element groups): two FMA chains in flight
        float s2[NQV][2];
#pragma unroll
        for (int r = 0; r < NQV; ++r) s2[r][0] = s2[r][1] = 0.f;
        const uint16_t* krow = Ks + pl * ROW;
#pragma unroll 8
        for (int c = 0; c < HD; c += 8) {
          const uint4 w = *(const uint4*)(krow + c);
          float kr[8];
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            kr[2 * i] = __uint_as_float(ww[i] << 16);
            kr[2 * i + 1] = __uint_as_float(ww[i] & 0xffff0000u);
          }
#pragma unroll
          for (int r = 0; r < NQV; ++r)
#pragma unroll
            for (int e = 0; e < 8; ++e) s2[r][(c >> 3) & 1] = fmaf(qs[r][c + e], kr[e], s2[r][(c >> 3) & 1]);
        }
#pragma unroll
        for (int r = 0; r < NQV; ++r) s[r] = s2[r][0] + s2[r][1];
      }
      float p[NQV];
#pragma unroll
      for (int r = 0; r < NQV; ++r) {
        p[r] = 0.f;
        if (r >= nqv) continue;
        float mv = -INFINITY;
        if (any) mv = rnd_dt(apply_chain(P, rnd_dt(s[r], P.dt_d1)) + mk[r], P.dt_m);
        float rm = mv;
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) rm = fmaxf(rm, __shfl_xor_sync(0xffffffffu, rm, sh));
        const float mnew = fmaxf(m[r], rm);
        if (mnew == -INFINITY) continue;
        if (any) p[r] = rnd_dt(expf(rnd_dt(mv - mnew, P.dt_sub)), P.dt_exp);
        float ps = p[r];
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, sh);
        const float sc = m[r] == -INFINITY ? 0.f : expf(m[r] - mnew);
        l[r] = l[r] * sc + ps;
#pragma unroll
        for (int e = 0; e < HPL; ++e) acc[r][e] *= sc;
        m[r] = mnew;
      }
      unsigned bits = valid;
      while (bits) {
        const int src = __ffs(bits) - 1;
        bits &= bits - 1;
        const uint16_t* vrow = Vs + (warp * 32 + src) * ROW + lane * HPL;
        float vr[HPL];
        load_row<uint16_t, HPL>(vrow, vr);
#pragma unroll
        for (int r = 0; r < NQV; ++r) {
          const float pj = __shfl_sync(0xffffffffu, p[r], src);
#pragma unroll
          for (int e = 0; e < HPL; ++e) acc[r][e] = fmaf(pj, vr[e], acc[r][e]);
        }
      }
    }
  }
  // merge warps (as attn_kernel)
#pragma unroll
  for (int r = 0; r < NQV; ++r) {
    if (lane == 0) { wm[warp][r] = m[r]; wl[warp][r] = l[r]; }
#pragma unroll
    for (int e = 0; e < HPL; ++e) wacc[warp][r][lane * HPL + e] = acc[r][e];
  }
  __syncthreads();
  const int64_t rows_total = (int64_t)P.B * P.nq * P.Sq;
  for (int e = threadIdx.x; e < nqv * HD; e += NW * 32) {
    int r = e / HD, d = e % HD;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][r]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < NW; ++w) {
        float sc = wm[w][r] == -INFINITY ? 0.f : expf(wm[w][r] - M);
        L += wl[w][r] * sc;
        A += wacc[w][r][d] * sc;
      }
    }
    int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
    int64_t row = ((int64_t)b * P.nq + h) * P.Sq + qi;
    if (P.splits == 1) {
      float o = L > 0.f ? A / L : 0.f;
      char* ob = dres(P.out, argtab);
      if (P.out_dt == KDT_F32) ((float*)ob)[row * HD + d] = o;
      else ((__nv_bfloat16*)ob)[row * HD + d] = __float2bfloat16_rn(o);
    } else {
      float* part = (float*)dres(P.part, argtab) + ((int64_t)split * rows_total + row) * (HD + 2);
      part[2 + d] = A;
      if (d == 0) { part[0] = M; part[1] = L; }
    }
  }
  merge_if_last(P, argtab, b, kh, i0, nqv);
}

__global__ void attn_combine_kernel(const __grid_constant__ AttnParams P, const uint64_t* __restrict__ argtab) {
  pdl_enter();
  const int64_t rows_total = (int64_t)P.B * P.nq * P.Sq;
  const int HD = P.hd;
  const float* part = (const float*)dres(P.part, argtab);
  char* ob = dres(P.out, argtab);
  for (int64_t row = blockIdx.x; row < rows_total; row += gridDim.x) {
    float M = -INFINITY;
    for (int s = 0; s < P.splits; ++s) M = fmaxf(M, part[((int64_t)s * rows_total + row) * (HD + 2)]);
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
      float L = 0.f, A = 0.f;
      if (M != -INFINITY) {
        for (int s = 0; s < P.splits; ++s) {
          const float* pp = part + ((int64_t)s * rows_total + row) * (HD + 2);
          if (pp[0] == -INFINITY) continue;
          float sc = expf(pp[0] - M);
          L += pp[1] * sc;
          A += pp[2 + d] * sc;
        }
      }
      float o = L > 0.f ? A / L : 0.f;
      if (P.out_dt == KDT_F32) ((float*)ob)[row * HD + d] = o;
      else ((__nv_bfloat16*)ob)[row * HD + d] = __float2bfloat16_rn(o);
    }
  }
}

// ---------------------------------------------------------------------------
// Decode attention on the tensor cores (mma.sync m16n8k16, bf16 in, f32
// accumulate).  One CTA per (batch * kv head, position split); its query
// vectors (the GQA group, at most 8) are the M rows of one 16-row tile.  The
// CTA walks its positions in chunks of TC_CH: the chunk's mask values go to
// shared memory, the 16-position steps with any unmasked position are staged
// (K and V rows, cp.async, double-buffered with the next chunk), and each of
// the 4 warps computes all scores of a step (S = Q K^T, 16 x 16) and then
// P V for its quarter of head_dim.  The printed score chain, mask, exp and
// roundings are replayed on the accumulator elements exactly as in the SIMT
// kernel.  P (f32) enters the P V product as a bf16 hi + lo pair, so the
// products keep ~16 significant bits (relative error ~2^-17, well inside the
// f32 tolerance of the attention output); every warp sees the same scores, so
// the per-row (max, sum) needs no cross-warp merge.
constexpr int TC_CH = 64;  // positions per staged chunk

__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// two f32 as a bf16 pair (round to nearest even): lo in bits 0-15
// bulk prefetch of [p, p + bytes) into L2 (16-byte aligned address and size)
__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float bf16_lo_f(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi_f(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

template <int HD>
__global__ void __launch_bounds__(128) attn_tc_kernel(const __grid_constant__ AttnParams P,
                                                     const uint64_t* __restrict__ argtab) {
  constexpr int ROW = HD + 8;            // padded smem row (bf16): rows 16 B apart in bank phase
  constexpr int KSTEPS = HD / 16;        // k-steps of the score product
  constexpr int NT = HD / 32;            // 8-dim output tiles per warp (a quarter of head_dim)
  static_assert(TC_CH == 4 * 16, "one 16-position score step per warp");
  extern __shared__ __align__(16) uint16_t tc_smem[];
  // K / V chunk buffers: two (double-buffered) when a CTA walks several chunks
  const int nbuf = (P.T + P.splits - 1) / P.splits > TC_CH ? 2 : 1;
  uint16_t* Kb = tc_smem;                          // [nbuf][TC_CH][ROW]
  uint16_t* Vb = tc_smem + nbuf * TC_CH * ROW;     // [nbuf][TC_CH][ROW]
  __shared__ float msk[2][8][TC_CH];
  __shared__ unsigned s_act[2];
  __shared__ float red_m[4][8], red_l[4][8];      // per-warp row max / sum of a chunk
  __shared__ uint32_t psm[2][8][TC_CH / 2 + 4];   // P hi / lo bf16 pairs, rows padded against bank conflicts
  // Q as bf16 parts: one for bf16 q; three (hi + mid + lo == q exactly) for f32 q
  __shared__ __align__(16) uint16_t qsm[3][8][HD + 8];
  // Before the dependency wait: pull this split's K/V rows towards L2.  A
  // prefetch returns nothing to the thread, so a row that the preceding
  // kernel is still writing (the new position) is read correctly after the wait.
  {
    const int64_t ch = (P.T + P.splits - 1) / P.splits;
    const int64_t p0 = blockIdx.x * ch, p1 = min((int64_t)P.T, p0 + ch);
    const int kb = blockIdx.z / P.nkv, kk = blockIdx.z % P.nkv;
    const uint16_t* kr = (const uint16_t*)dres(P.k.p, argtab) + kb * P.k.stride[0] + kk * P.k.stride[1];
    const uint16_t* vr = (const uint16_t*)dres(P.v.p, argtab) + kb * P.v.stride[0] + kk * P.v.stride[1];
    if (P.k.stride[2] == HD && P.v.stride[2] == HD) {  // contiguous rows: 16 KB pieces
      const int64_t bytes = (p1 - p0) * HD * 2;
      for (int64_t i = threadIdx.x; i * 16384 < bytes; i += 128) {
        const uint32_t n = (uint32_t)min((int64_t)16384, bytes - i * 16384);
        l2_prefetch_bulk((const char*)(kr + p0 * HD) + i * 16384, n);
        l2_prefetch_bulk((const char*)(vr + p0 * HD) + i * 16384, n);
      }
    } else {
      for (int64_t i = threadIdx.x; i < p1 - p0; i += 128) {
        l2_prefetch_bulk(kr + (p0 + i) * P.k.stride[2], HD * 2);
        l2_prefetch_bulk(vr + (p0 + i) * P.v.stride[2], HD * 2);
      }
    }
  }
  pdl_enter();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int bk = blockIdx.z;
  const int b = bk / P.nkv, kh = bk % P.nkv;
  const int nqv = P.Sq * P.group;  // decode: one query tile holds every query vector of the group
  const int split = blockIdx.x;
  const int64_t chunk = (P.T + P.splits - 1) / P.splits;
  const int64_t t0 = split * chunk, t1 = min((int64_t)P.T, t0 + chunk);
  const char* qb = dres(P.q.p, argtab);
  const uint16_t* kbase = (const uint16_t*)dres(P.k.p, argtab) + b * P.k.stride[0] + kh * P.k.stride[1];
  const uint16_t* vbase = (const uint16_t*)dres(P.v.p, argtab) + b * P.v.stride[0] + kh * P.v.stride[1];
  const char* mb = dres(P.mask.p, argtab);
  const int qp0 = mask_qpos0(P, argtab);
  auto qrow = [&](int r, int& qi, int& h) {
    qi = r / P.group;
    h = kh * P.group + r % P.group;
  };
  // Q through shared memory; A fragments are read per k-step: rows >= nqv are
  // zero, and rows 8-15 of the 16-row tile (a1, a3) are always zero
  const bool qf32 = P.q.dt == KDT_F32;
  const int qparts = qf32 ? 3 : 1;
  __shared__ int64_t qoff_s[8], moff_s[8];
  if (threadIdx.x < 8) {
    const int r = threadIdx.x < nqv ? threadIdx.x : 0;
    int qi, h;
    qrow(r, qi, h);
    qoff_s[threadIdx.x] = b * P.q.stride[0] + h * P.q.stride[1] + qi * P.q.stride[2];
    moff_s[threadIdx.x] = b * P.mask.stride[0] + h * P.mask.stride[1] + qi * P.mask.stride[2];
  }
  for (int e = threadIdx.x; e < 3 * 8 * (HD + 8) / 8; e += 128) ((uint4*)&qsm[0][0][0])[e] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  const int64_t qs3 = P.q.stride[3];
  // all of this thread's query loads in flight before the shared stores
  float qv[8 * HD / 128];
#pragma unroll
  for (int u = 0; u < 8 * HD / 128; ++u) {
    const int e = threadIdx.x + 128 * u;
    qv[u] = 0.f;
    if (e < nqv * HD) {
      const int64_t o = qoff_s[e / HD] + (e % HD) * qs3;
      qv[u] = qf32 ? ((const float*)qb)[o] : __uint_as_float((uint32_t)((const uint16_t*)qb)[o]);
    }
  }
#pragma unroll
  for (int u = 0; u < 8 * HD / 128; ++u) {
    const int e = threadIdx.x + 128 * u;
    if (e >= nqv * HD) break;
    const int r = e / HD, c = e % HD;
    if (qf32) {
      const float q = qv[u];
      const __nv_bfloat16 hi = __float2bfloat16_rn(q);
      const float r1 = q - __bfloat162float(hi);
      const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
      const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
      qsm[0][r][c] = __bfloat16_as_ushort(hi);
      qsm[1][r][c] = __bfloat16_as_ushort(mid);
      qsm[2][r][c] = __bfloat16_as_ushort(lo);
    } else {
      qsm[0][r][c] = (uint16_t)__float_as_uint(qv[u]);
    }
  }
  const uint32_t qsa = (uint32_t)__cvta_generic_to_shared(&qsm[0][g][2 * t]);
  constexpr uint32_t QPART = 8 * (HD + 8) * 2;  // bytes between Q parts
  // stage chunk c0 into buffer buf: mask values, active steps, K/V rows of active steps
  // staging of a chunk, in two halves around a barrier the caller places:
  // mask values first, then (once they are visible) the K/V rows of active steps
  auto stage_mask = [&](int64_t c0, int buf) {
    for (int e = threadIdx.x; e < nqv * TC_CH; e += 128) {
      const int r = e / TC_CH, j = e % TC_CH;
      float v = -INFINITY;
      if (c0 + j < t1) v = mask_at(P, mb, moff_s[r], c0 + j, qp0);
      msk[buf][r][j] = v;
    }
    if (threadIdx.x == 0) s_act[buf] = 0u;
  };
  // active 16-position steps of a staged mask (after a barrier; one follows)
  auto stage_active = [&](int buf) {
    if (threadIdx.x < TC_CH) {
      bool any = false;
      for (int r = 0; r < nqv; ++r) any |= msk[buf][r][threadIdx.x] > P.mask_skip;
      if (any) atomicOr(&s_act[buf], 1u << (threadIdx.x / 16));
    }
  };
  // K/V rows of the steps in `act` (one cp.async group)
  auto stage_copy = [&](int64_t c0, int buf, unsigned act) {
    constexpr int SEGS = HD / 8;  // 16-byte pieces per row
    for (int q = threadIdx.x; q < TC_CH * SEGS; q += 128) {
      const int rr = q / SEGS, sg = q % SEGS;
      if (!((act >> (rr / 16)) & 1u)) continue;
      uint16_t* kd = Kb + ((size_t)buf * TC_CH + rr) * ROW + sg * 8;
      uint16_t* vd = Vb + ((size_t)buf * TC_CH + rr) * ROW + sg * 8;
      if (c0 + rr < t1) {
        cp_async16(kd, kbase + (c0 + rr) * P.k.stride[2] + sg * 8);
        cp_async16(vd, vbase + (c0 + rr) * P.v.stride[2] + sg * 8);
      } else {  // past the split's last position: zeros (never NaN into P V)
        *(uint4*)kd = make_uint4(0, 0, 0, 0);
        *(uint4*)vd = make_uint4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[n][i] = 0.f;
  const uint32_t kb_s = (uint32_t)__cvta_generic_to_shared(Kb), vb_s = (uint32_t)__cvta_generic_to_shared(Vb);
  int buf = 0;
  // the first chunk's mask values load together with the queries above; then
  // only the K/V rows of its active steps (a CTA whose positions are all masked,
  // as most are in a sliding-window layer, reads no K/V)
  if (t0 < t1) stage_mask(t0, 0);
  __syncthreads();
  if (t0 < t1) stage_active(0);
  __syncthreads();
  if (t0 < t1) stage_copy(t0, 0, s_act[0]);
  for (int64_t c0 = t0; c0 < t1; c0 += TC_CH, buf ^= 1) {
    const bool more = c0 + TC_CH < t1;
    if (more) {
      stage_mask(c0 + TC_CH, buf ^ 1);  // next chunk in flight while this one is computed
      __syncthreads();
      stage_active(buf ^ 1);
      __syncthreads();
      stage_copy(c0 + TC_CH, buf ^ 1, s_act[buf ^ 1]);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const unsigned act = s_act[buf];
    // scores of this warp's 16-position step (S = Q K^T, 16 x 16), four
    // independent accumulator sets (k-step mod 4) so four mma chains are in flight
    const int s0 = warp * 16;
    const bool mine = (act >> warp) & 1u;
    float mv[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    if (mine) {
      float sp[4][2][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int i = 0; i < 4; ++i) sp[a][0][i] = sp[a][1][i] = 0.f;
      const int mi = lane >> 3, ri = lane & 7;
      const uint32_t rowaddr =
          kb_s + (uint32_t)((((size_t)buf * TC_CH + s0 + ri + 8 * (mi >> 1)) * ROW + 8 * (mi & 1)) * 2);
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        uint32_t bf[4];
        ldsm_x4(rowaddr + 32u * kk, bf);
        for (int qp = 0; qp < qparts; ++qp) {
          uint32_t a0, a2;
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(a0) : "r"(qsa + qp * QPART + 32u * kk));
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(a2) : "r"(qsa + qp * QPART + 32u * kk + 16u));
          mma_bf16(sp[kk & 3][0], a0, 0u, a2, 0u, bf[0], bf[1]);
          mma_bf16(sp[kk & 3][1], a0, 0u, a2, 0u, bf[2], bf[3]);
        }
      }
      // chain and mask on this thread's row-g elements (rows g + 8 are padding:
      // at most 8 query vectors)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int tile = q >> 1, i = q & 1;
        const float acc = (sp[0][tile][i] + sp[1][tile][i]) + (sp[2][tile][i] + sp[3][tile][i]);
        const int j = s0 + 8 * tile + 2 * t + i;
        const float mk = msk[buf][g][j];
        if (g < nqv && mk > P.mask_skip)
          mv[q] = rnd_dt(apply_chain(P, rnd_dt(acc, P.dt_d1)) + mk, P.dt_m);
      }
    }
    float rmax = fmaxf(fmaxf(mv[0], mv[1]), fmaxf(mv[2], mv[3]));
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 1));
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 2));
    if (t == 0) red_m[warp][g] = rmax;
    __syncthreads();
    // the chunk's row maximum, the same in every warp
    const float mnew = fmaxf(fmaxf(m[0], fmaxf(red_m[0][g], red_m[1][g])), fmaxf(red_m[2][g], red_m[3][g]));
    float pv[4];
    float ps = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      pv[q] = 0.f;
      if (mnew != -INFINITY && mv[q] != -INFINITY) pv[q] = rnd_dt(expf(rnd_dt(mv[q] - mnew, P.dt_sub)), P.dt_exp);
      ps += pv[q];
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    if (t == 0) red_l[warp][g] = ps;
    // P of this step as bf16 hi / lo pairs for the P V product of every warp
#pragma unroll
    for (int tile = 0; tile < 2; ++tile) {
      const uint32_t hi = pack_bf16(pv[2 * tile], pv[2 * tile + 1]);
      const uint32_t lo = pack_bf16(pv[2 * tile] - bf16_lo_f(hi), pv[2 * tile + 1] - bf16_hi_f(hi));
      psm[0][g][8 * warp + 4 * tile + t] = hi;
      psm[1][g][8 * warp + 4 * tile + t] = lo;
    }
    __syncthreads();
    if (mnew != -INFINITY) {
      const float csum = (red_l[0][g] + red_l[1][g]) + (red_l[2][g] + red_l[3][g]);
      const float scl = m[0] == -INFINITY ? 0.f : expf(m[0] - mnew);
      l[0] = l[0] * scl + csum;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        o[n][0] *= scl;
        o[n][1] *= scl;
      }
      m[0] = mnew;
    }
    // O[:, warp quarter] += P V over the chunk's active steps
#pragma unroll 1
    for (int st = 0; st < TC_CH / 16; ++st) {
      if (!((act >> st) & 1u)) continue;
      const uint32_t ah0 = psm[0][g][8 * st + t], ah2 = psm[0][g][8 * st + 4 + t];
      const uint32_t al0 = psm[1][g][8 * st + t], al2 = psm[1][g][8 * st + 4 + t];
      const int mi = lane >> 3, ri = lane & 7;
      const uint32_t rowaddr = vb_s + (uint32_t)((((size_t)buf * TC_CH + 16 * st + ri + 8 * (mi & 1)) * ROW +
                                                  warp * (HD / 4) + 8 * (mi >> 1)) * 2);
#pragma unroll
      for (int n = 0; n < NT; n += 2) {
        uint32_t bf[4];
        ldsm_x4_t(rowaddr + 32u * (n / 2), bf);
        mma_bf16(o[n], ah0, 0u, ah2, 0u, bf[0], bf[1]);
        mma_bf16(o[n], al0, 0u, al2, 0u, bf[0], bf[1]);
        mma_bf16(o[n + 1], ah0, 0u, ah2, 0u, bf[2], bf[3]);
        mma_bf16(o[n + 1], al0, 0u, al2, 0u, bf[2], bf[3]);
      }
    }
    __syncthreads();  // red / psm and this buffer are rewritten by the next chunk
  }
  // results: rows g and g + 8 of this warp's quarter of head_dim
  const int64_t rows_total = (int64_t)P.B * P.nq * P.Sq;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = g + 8 * hr;
    if (r >= nqv) continue;
    int qi, h;
    qrow(r, qi, h);
    const int64_t row = ((int64_t)b * P.nq + h) * P.Sq + qi;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int d = warp * (HD / 4) + 8 * n + 2 * t + e;
        const float A = o[n][2 * hr + e];
        if (P.splits == 1) {
          const float v = l[hr] > 0.f ? A / l[hr] : 0.f;
          char* ob = dres(P.out, argtab);
          if (P.out_dt == KDT_F32) ((float*)ob)[row * HD + d] = v;
          else ((__nv_bfloat16*)ob)[row * HD + d] = __float2bfloat16_rn(v);
        } else {
          float* part = (float*)dres(P.part, argtab) + ((int64_t)split * rows_total + row) * (HD + 2);
          part[2 + d] = A;
          if (d == 0) {
            part[0] = m[hr];
            part[1] = l[hr];
          }
        }
      }
  }
  merge_if_last(P, argtab, b, kh, 0, nqv);
}

// ---------------------------------------------------------------------------
// Decode attention with bulk-copy staged K/V (use_tc 3).  A decode step reads
// each cached K/V row once and does ~2 flops per byte, so the kernel is built
// for latency and for many short CTAs: 4 warps, a split of DEC_CH (64)
// positions per CTA (more, in chunks of DEC_CH, when a cache is longer than 64
// splits), so a layer is one or two waves.  Before the dependency wait a CTA
// asks L2 for its split's rows.  After it, the CTA loads the chunk's mask
// values and its query vectors (registers, lane-owned dims), finds the live
// positions (any query's mask above mask_skip), and one thread copies just
// those K / V rows into shared memory with cp.async.bulk; a chunk with no live
// position (most chunks of a sliding-window layer) reads no K / V at all.
// Scores are f32 on the CUDA cores (f32 queries need no split): each warp
// takes 32 / NQ positions at a time, every lane accumulating its dims of all
// of them for every query vector, and one reduce-scatter across the lanes
// (16 + 8 + 4 + 2 + 1 shuffles) leaves lane l holding the score of position
// l / NQ for query l % NQ; the printed chain, mask and roundings follow.  The
// chunk softmax runs over the scores in shared memory and each warp
// accumulates P V over its positions; the warps' contexts are summed through
// shared memory.  Splits are merged by the last CTA of a (batch, kv head) to
// arrive, which copies every split's partial row block into shared memory
// with one bulk copy each (rows padded to 16-byte multiples for that).
constexpr int DEC_THREADS = 128;
constexpr int DEC_CH = 64;  // positions per staged chunk (and per split when it fits)

__device__ __forceinline__ uint32_t dec_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool dec_mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = dec_smem_u32(bar);
  for (uint32_t i = 0; i < (1u << 22); ++i) {  // bounded: a copy that never lands is reported, not waited for
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void dec_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dec_smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(dec_smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void dec_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(dec_smem_u32(bar)), "r"(bytes)
               : "memory");
}

// floats per partial row of the staged decode kernel: (max, sum, 2 pad, context[HD]),
// a 16-byte multiple so that a (split, batch, kv head) block is one bulk copy
__host__ __device__ constexpr int dec_part_stride(int hd) { return hd + 4; }

// reduce-scatter of 32 values across a warp: lane l returns the warp-wide sum of v[l]
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16, n = 32; o >= 1; o >>= 1, n >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

template <int HD, int NQ>
__global__ void __launch_bounds__(DEC_THREADS) attn_dec_kernel(const __grid_constant__ AttnParams P,
                                                               const uint64_t* __restrict__ argtab) {
  constexpr int VPL = HD / 32;        // consecutive dims of a row per lane
  constexpr int NWARP = DEC_THREADS / 32;
  constexpr int PG = 32 / NQ;         // positions a warp scores at a time (PG * NQ == 32)
  constexpr int PS = dec_part_stride(HD);
  extern __shared__ __align__(128) unsigned char dec_smem[];
  uint16_t* Kb = (uint16_t*)dec_smem;                 // [DEC_CH][HD]
  uint16_t* Vb = Kb + DEC_CH * HD;                    // [DEC_CH][HD]
  float* msk = (float*)(Vb + DEC_CH * HD);            // [NQ][DEC_CH]
  float* sc = msk + NQ * DEC_CH;                      // [NQ][DEC_CH] scores, then probabilities
  __shared__ __align__(8) uint64_t bar;
  __shared__ float s_m[NQ], s_l[NQ], s_scl[NQ];
  __shared__ int s_lo[2], s_hi[2];
  __shared__ int64_t s_qoff[NQ], s_moff[NQ];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bk = blockIdx.y, b = bk / P.nkv, kh = bk % P.nkv;
  const int nqv = P.group;  // Sq == 1: one query vector per head of the group
  // a computed mask needs only the position (a graph parameter, never written
  // by a plan kernel): read it before the dependency wait
  const int qp0 = mask_qpos0(P, argtab);
  int64_t t0 = (int64_t)blockIdx.x * P.dec_per_split, t1 = min((int64_t)P.T, t0 + P.dec_per_split);
  if (P.dec_live_splits) {
    // the live positions [lo, hi] spread evenly over the splits
    const int64_t lo = max((int64_t)0, (int64_t)qp0 + P.mask_lt);
    const int64_t hi = min((int64_t)P.T - 1, (int64_t)qp0 + P.mask_gt);
    const int64_t n = max((int64_t)0, hi - lo + 1), per = (n + P.splits - 1) / P.splits;
    t0 = min(hi + 1, lo + (int64_t)blockIdx.x * per);
    t1 = min(hi + 1, t0 + per);
    if (n == 0) t0 = t1 = 0;
  }
  const uint16_t* kbase = (const uint16_t*)dres(P.k.p, argtab) + b * P.k.stride[0] + kh * P.k.stride[1];
  const uint16_t* vbase = (const uint16_t*)dres(P.v.p, argtab) + b * P.v.stride[0] + kh * P.v.stride[1];
  const int64_t ks = P.k.stride[2], vs = P.v.stride[2];
  const bool dense = ks == HD && vs == HD;
  // before the dependency wait: the split's rows towards L2 (rows before the new
  // position were written by earlier steps; a prefetch returns nothing, so the
  // new row is read correctly after the wait)
  if (t0 < t1) {
    if (dense) {
      const int64_t bytes = (t1 - t0) * HD * 2;
      for (int64_t i = threadIdx.x; i * 8192 < bytes; i += DEC_THREADS) {
        const uint32_t n = (uint32_t)min((int64_t)8192, bytes - i * 8192);
        l2_prefetch_bulk((const char*)(kbase + t0 * HD) + i * 8192, n);
        l2_prefetch_bulk((const char*)(vbase + t0 * HD) + i * 8192, n);
      }
    } else {
      for (int64_t i = threadIdx.x; i < t1 - t0; i += DEC_THREADS) {
        l2_prefetch_bulk(kbase + (t0 + i) * ks, HD * 2);
        l2_prefetch_bulk(vbase + (t0 + i) * vs, HD * 2);
      }
    }
  }
  // the following GEMVs' weights towards L2 (never written by a plan kernel):
  // this CTA's slice of each region, in region order
  {
    const int64_t nct = (int64_t)gridDim.x * gridDim.y, me = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
    for (int h = 0; h < P.nhint; ++h) {
      const int64_t per = ((P.hint_bytes[h] + nct - 1) / nct + 15) & ~(int64_t)15;
      const int64_t lo = me * per, hi = min(P.hint_bytes[h], lo + per);
      const char* base = dres(P.hint[h], argtab);
      for (int64_t o = lo + (int64_t)threadIdx.x * 4096; o < hi; o += (int64_t)DEC_THREADS * 4096)
        l2_prefetch_bulk(base + o, (uint32_t)min((int64_t)4096, hi - o));
    }
  }
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(dec_smem_u32(&bar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < NQ) {
    const int r = threadIdx.x < nqv ? threadIdx.x : 0;
    const int h = kh * P.group + r;
    s_qoff[threadIdx.x] = b * P.q.stride[0] + h * P.q.stride[1];
    s_moff[threadIdx.x] = b * P.mask.stride[0] + h * P.mask.stride[1];
    s_m[threadIdx.x] = -INFINITY;
    s_l[threadIdx.x] = 0.f;
  }
  __syncthreads();
  pdl_enter();
  unsigned* status = P.has_status ? (unsigned*)dres(P.status, argtab) : nullptr;
  const char* mb = dres(P.mask.p, argtab);
  // queries: lane-owned dims of every query vector, f32
  float q[NQ][VPL];
  {
    const char* qb = dres(P.q.p, argtab);
    const int64_t qs3 = P.q.stride[3];
#pragma unroll
    for (int r = 0; r < NQ; ++r)
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        q[r][i] = r < nqv ? ld_any(qb, s_qoff[r] + (int64_t)(lane * VPL + i) * qs3, P.q.dt) : 0.f;
  }
  float acc[NQ][VPL];
#pragma unroll
  for (int r = 0; r < NQ; ++r)
#pragma unroll
    for (int i = 0; i < VPL; ++i) acc[r][i] = 0.f;
  uint32_t phase = 0;
  bool ok = true;
  if (threadIdx.x == 0) {
    s_lo[0] = DEC_CH;
    s_hi[0] = -1;
  }
  for (int64_t c0 = t0, k = 0; c0 < t1; c0 += DEC_CH, ++k) {
    const int n = (int)min((int64_t)DEC_CH, t1 - c0);
    const int kp = (int)(k & 1);
    __syncthreads();  // the previous chunk is done with every buffer; this chunk's s_lo / s_hi reset
    // mask values of the chunk and its live positions [lo, hi]
    int lo = DEC_CH, hi = -1;
    for (int e = threadIdx.x; e < NQ * DEC_CH; e += DEC_THREADS) {
      const int r = e / DEC_CH, j = e % DEC_CH;
      float v = -INFINITY;
      if (r < nqv && j < n) v = mask_at(P, mb, s_moff[r], c0 + j, qp0);
      msk[e] = v;
      if (v > P.mask_skip) {
        lo = min(lo, j);
        hi = max(hi, j);
      }
    }
    if (hi >= 0) {
      atomicMin(&s_lo[kp], lo);
      atomicMax(&s_hi[kp], hi);
    }
    __syncthreads();
    lo = s_lo[kp];
    hi = s_hi[kp];
    if (threadIdx.x == 0) {  // the next chunk's (last read before the barrier above)
      s_lo[kp ^ 1] = DEC_CH;
      s_hi[kp ^ 1] = -1;
    }
    if (hi < 0) continue;  // nothing live in this chunk: no K / V read (uniform)
    const int nl = hi - lo + 1;
    if (threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      dec_expect(&bar, (uint32_t)(2 * nl * HD * 2));
      if (dense) {
        dec_bulk(Kb + lo * HD, kbase + (c0 + lo) * HD, (uint32_t)(nl * HD * 2), &bar);
        dec_bulk(Vb + lo * HD, vbase + (c0 + lo) * HD, (uint32_t)(nl * HD * 2), &bar);
      } else {
        for (int j = lo; j <= hi; ++j) {
          dec_bulk(Kb + j * HD, kbase + (c0 + j) * ks, HD * 2, &bar);
          dec_bulk(Vb + j * HD, vbase + (c0 + j) * vs, HD * 2, &bar);
        }
      }
    }
    bool landed = dec_mbar_wait(&bar, phase);
    if (!landed) landed = dec_mbar_wait(&bar, phase);  // once more: the copy may still land
    phase ^= 1u;
    ok = __syncthreads_and(ok && landed) != 0;
    if (!ok) {
      if (status && threadIdx.x == 0) atomicOr(status, 32u);
      break;
    }
    // scores: warp w takes positions lo + PG g .. + PG - 1 for g = w, w + NWARP, ...
    for (int g0 = lo + warp * PG; g0 <= hi; g0 += NWARP * PG) {
      float part[32];
#pragma unroll
      for (int p = 0; p < PG; ++p) {
        const int j = g0 + p;
        float kv[VPL];
        if (j <= hi) load_row<uint16_t, VPL>(Kb + j * HD + lane * VPL, kv);
#pragma unroll
        for (int r = 0; r < NQ; ++r) {
          float s = 0.f;
          if (j <= hi) {
#pragma unroll
            for (int i = 0; i < VPL; ++i) s = fmaf(q[r][i], kv[i], s);
          }
          part[p * NQ + r] = s;
        }
      }
      const float dot = warp_reduce_scatter32(part, lane);
      const int j = g0 + lane / NQ, r = lane % NQ;
      if (j <= hi && r < nqv) {
        const float mk = msk[r * DEC_CH + j];
        sc[r * DEC_CH + j] = mk > P.mask_skip ? rnd_dt(apply_chain(P, rnd_dt(dot, P.dt_d1)) + mk, P.dt_m) : -INFINITY;
      }
    }
    __syncthreads();
    // chunk softmax: warp r reduces row r over [lo, hi]
    for (int r = warp; r < nqv; r += NWARP) {
      float mx = -INFINITY;
      for (int j = lo + lane; j <= hi; j += 32) mx = fmaxf(mx, sc[r * DEC_CH + j]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = s_m[r], mnew = fmaxf(mold, mx);
      float sum = 0.f;
      for (int j = lo + lane; j <= hi; j += 32) {
        const float s = sc[r * DEC_CH + j];
        float p = 0.f;
        if (mnew != -INFINITY && s != -INFINITY) p = rnd_dt(expf(rnd_dt(s - mnew, P.dt_sub)), P.dt_exp);
        sc[r * DEC_CH + j] = p;
        sum += p;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        const float scl = mnew == -INFINITY ? 1.f : (mold == -INFINITY ? 0.f : expf(mold - mnew));
        s_scl[r] = scl;
        s_l[r] = s_l[r] * scl + sum;
        s_m[r] = mnew;
      }
    }
    __syncthreads();
    // P V: warp w takes positions lo + w, lo + w + NWARP, ...
#pragma unroll
    for (int r = 0; r < NQ; ++r) {
      const float scl = r < nqv ? s_scl[r] : 1.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i) acc[r][i] *= scl;
    }
    int j = lo + warp;
    for (; j + 3 * NWARP <= hi; j += 4 * NWARP) {  // four positions in flight
      float vv[4][VPL], p[4][NQ];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        load_row<uint16_t, VPL>(Vb + (j + u * NWARP) * HD + lane * VPL, vv[u]);
#pragma unroll
        for (int r = 0; r < NQ; ++r) p[u][r] = r < nqv ? sc[r * DEC_CH + j + u * NWARP] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int r = 0; r < NQ; ++r)
#pragma unroll
          for (int i = 0; i < VPL; ++i) acc[r][i] = fmaf(p[u][r], vv[u][i], acc[r][i]);
    }
    for (; j <= hi; j += NWARP) {
      float vv[VPL];
      load_row<uint16_t, VPL>(Vb + j * HD + lane * VPL, vv);
#pragma unroll
      for (int r = 0; r < NQ; ++r) {
        const float p = r < nqv ? sc[r * DEC_CH + j] : 0.f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) acc[r][i] = fmaf(p, vv[i], acc[r][i]);
      }
    }
  }
  // the warps' contexts summed through shared memory (the chunk buffers are free)
  __syncthreads();
  float* red = (float*)dec_smem;  // [NWARP][NQ][HD]
#pragma unroll
  for (int r = 0; r < NQ; ++r)
#pragma unroll
    for (int i = 0; i < VPL; ++i) red[(warp * NQ + r) * HD + lane * VPL + i] = acc[r][i];
  __syncthreads();
  const int64_t rows_total = (int64_t)P.B * P.nq;
  const int64_t row0 = (int64_t)b * P.nq + kh * P.group;  // this head group's first output row
  float* part = P.splits > 1 ? (float*)dres(P.part, argtab) : nullptr;
  for (int e = threadIdx.x; e < nqv * HD; e += DEC_THREADS) {
    const int r = e / HD, d = e % HD;
    float A = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) A += red[(w * NQ + r) * HD + d];
    if (P.splits == 1) {
      const float l = s_l[r];
      const float v = l > 0.f ? A / l : 0.f;
      char* ob = dres(P.out, argtab);
      if (P.out_dt == KDT_F32) ((float*)ob)[(row0 + r) * HD + d] = v;
      else ((__nv_bfloat16*)ob)[(row0 + r) * HD + d] = __float2bfloat16_rn(v);
    } else {
      float* pr = part + ((int64_t)blockIdx.x * rows_total + row0 + r) * PS;
      pr[4 + d] = A;
      if (d == 0) {
        pr[0] = s_m[r];
        pr[1] = s_l[r];
      }
    }
  }
  if (P.splits == 1) return;
  // the last split to arrive merges: every split's block of partial rows comes
  // in with one bulk copy (issued by the four warps in turn) into shared memory
  __shared__ int s_last;
  __shared__ float s_w[ATTN_MERGE_MAX_SPLITS][NQ];
  __shared__ float s_tot[NQ];
  __syncthreads();  // every thread's partial stores before thread 0's release
  unsigned* ctr = (unsigned*)dres(P.counters, argtab) + bk;
  if (threadIdx.x == 0) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
    s_last = old == (unsigned)(P.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  const int S = P.splits;
  float* pm = (float*)dec_smem;  // [S][nqv][PS]
  const uint32_t blk = (uint32_t)(nqv * PS * 4);
  if (threadIdx.x == 0) {
    // the partials were written by other CTAs (generic proxy, made visible by
    // the acquire above); the async-proxy reads below are ordered after it
    asm volatile("fence.proxy.async.global;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    dec_expect(&bar, blk * (uint32_t)S);
  }
  __syncthreads();
  for (int sp = threadIdx.x; sp < S; sp += DEC_THREADS)
    dec_bulk(pm + (size_t)sp * nqv * PS, part + ((int64_t)sp * rows_total + row0) * PS, blk, &bar);
  bool landed = dec_mbar_wait(&bar, phase);
  if (!landed) landed = dec_mbar_wait(&bar, phase);
  if (!__syncthreads_and(landed)) {
    if (status && threadIdx.x == 0) atomicOr(status, 64u);
    if (threadIdx.x == 0) *ctr = 0u;
    return;
  }
  // the splits' weights exp(m_s - M) per query vector, one warp per vector
  for (int r = warp; r < nqv; r += NWARP) {
    float M = -INFINITY;
    for (int sp = lane; sp < S; sp += 32) M = fmaxf(M, pm[(sp * nqv + r) * PS]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int sp = lane; sp < S; sp += 32) {
      const float m = pm[(sp * nqv + r) * PS];
      const float w = (M == -INFINITY || m == -INFINITY) ? 0.f : expf(m - M);
      s_w[sp][r] = w;
      L += w == 0.f ? 0.f : pm[(sp * nqv + r) * PS + 1] * w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) s_tot[r] = L;
  }
  __syncthreads();
  char* ob = dres(P.out, argtab);
  for (int e = threadIdx.x; e < nqv * HD; e += DEC_THREADS) {
    const int r = e / HD, d = e % HD;
    float A = 0.f;
    for (int sp = 0; sp < S; ++sp) A += pm[(sp * nqv + r) * PS + 4 + d] * s_w[sp][r];
    const float L = s_tot[r];
    const float v = L > 0.f ? A / L : 0.f;
    if (P.out_dt == KDT_F32) ((float*)ob)[(row0 + r) * HD + d] = v;
    else ((__nv_bfloat16*)ob)[(row0 + r) * HD + d] = __float2bfloat16_rn(v);
  }
  if (threadIdx.x == 0) *ctr = 0u;  // ready for the next launch
}

// ---------------------------------------------------------------------------
// Prefill attention on the tensor cores (FA2-style, mma.sync m16n8k16 bf16 ->
// f32).  One CTA per (batch * kv head, 64 query vectors): query vector
// r = qi * group + gi of the tile's query positions, so the GQA group shares
// every staged K/V row.  8 warps: warp w owns rows 16 (w & 3) .. + 15 and
// half (w >> 2) of head_dim.  The two warps of a row group share its
// rows; each scores half of a 64-position chunk (S = Q K^T), they exchange
// their row maxima and P fragments through shared memory (a 64-thread named
// barrier per pair), and apply the same rescaling, so their online-softmax
// states agree.  One pass over the CTA's mask rows first marks the
// 64-position chunks holding any position above mask_skip (the causal upper
// triangle and positions outside a sliding window drop out); only those are
// staged, K / V with cp.async, double-buffered.  Tiles are issued longest
// first (the last query positions see the most chunks).  K (with the mask
// tile) is double-buffered; V has one buffer, restaged after each P V so that
// an f32 query tile still fits beside the K, V and mask tiles at head_dim 256.
// P enters P V, and f32 queries the score product, as the exact bf16 split
// hi + mid + lo of the f32 value (P V is the printed f32 x bf16 product).
//
// FAST: the additive mask is f32 with 16-byte aligned rows and the score
// chain has a closed form with f32 softmax arithmetic (the printed Gemma and
// GPT-2 blocks): each chunk's mask tile is staged into shared memory with K / V
// and the per-score work is a few register operations.  Otherwise the printed
// chain and roundings are replayed per score with the mask read from memory.
constexpr int PF_CH = 64;   // positions per staged chunk
constexpr int PF_ROWS = 64; // query vectors per CTA
constexpr int PF_MROW = PF_CH + 4;  // padded f32 row of a staged mask tile
constexpr int PF_LIVE_WORDS = 32;   // live-chunk bitmap: T <= 32 * 32 * 64 positions

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// the two warps (64 threads) of row group rg: named barrier 1 + rg
__device__ __forceinline__ void pair_sync(int rg) { asm volatile("bar.sync %0, 64;" ::"r"(1 + rg) : "memory"); }

template <int HD, bool FAST>
__global__ void __launch_bounds__(256, 1) attn_tc_prefill_kernel(const __grid_constant__ AttnParams P,
                                                                 const uint64_t* __restrict__ argtab) {
  constexpr int ROW = HD + 8;           // padded bf16 row of K / V / bf16 Q
  constexpr int QROWF = HD + 4;         // padded f32 row of an f32 Q
  constexpr int KSTEPS = HD / 16;
  constexpr int NTO = HD / 16;          // 8-dim output tiles per warp (half of head_dim)
  extern __shared__ __align__(16) unsigned char pf_smem[];
  uint16_t* Kb = (uint16_t*)pf_smem;                    // [2][PF_CH][ROW]
  uint16_t* Vb = Kb + 2 * PF_CH * ROW;                  // [PF_CH][ROW]
  float* Ms = (float*)(Vb + PF_CH * ROW);               // FAST: [2][PF_ROWS][PF_MROW]
  unsigned char* Qs = (unsigned char*)(Ms + (FAST ? 2 * PF_ROWS * PF_MROW : 0));  // bf16 [64][ROW] / f32 [64][QROWF]
  __shared__ int64_t qoff_s[PF_ROWS], moff_s[PF_ROWS];
  __shared__ unsigned live_s[PF_LIVE_WORDS];
  __shared__ float pm_s[2][PF_ROWS];                  // per-half row maxima (then sums)
  __shared__ float pf_s[4][2][2][8][32];              // P values [row group][half][k-step][element][lane]
  pdl_enter();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rg = warp & 3, dh = warp >> 2;
  const int bk = blockIdx.z, b = bk / P.nkv, kh = bk % P.nkv;
  const int QT = PF_ROWS / P.group;  // query positions per CTA
  const int i0 = (int)(gridDim.y - 1 - blockIdx.y) * QT;  // longest tiles first
  const int nrows = min(QT, P.Sq - i0) * P.group;
  const bool qf32 = P.q.dt == KDT_F32;
  const char* qb = dres(P.q.p, argtab);
  const uint16_t* kbase = (const uint16_t*)dres(P.k.p, argtab) + b * P.k.stride[0] + kh * P.k.stride[1];
  const uint16_t* vbase = (const uint16_t*)dres(P.v.p, argtab) + b * P.v.stride[0] + kh * P.v.stride[1];
  const char* mb = dres(P.mask.p, argtab);
  const int qp0 = mask_qpos0(P, argtab);
  const float* mf = (const float*)mb;
  if (threadIdx.x < PF_ROWS) {
    const int r = threadIdx.x < nrows ? threadIdx.x : 0;
    const int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
    qoff_s[threadIdx.x] = b * P.q.stride[0] + h * P.q.stride[1] + qi * P.q.stride[2];
    moff_s[threadIdx.x] = b * P.mask.stride[0] + h * P.mask.stride[1] + qi * P.mask.stride[2];
  }
  if (threadIdx.x < PF_LIVE_WORDS) live_s[threadIdx.x] = 0u;
  __syncthreads();
  // Q -> shared (rows >= nrows zero); eight loads in flight per thread before
  // their shared stores
  for (int e0 = threadIdx.x; e0 < PF_ROWS * HD; e0 += 8 * 256) {
    uint32_t val[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + 256 * u, r = e / HD, c = e % HD;
      val[u] = 0u;
      if (r < nrows) {
        const int64_t o = qoff_s[r] + c * P.q.stride[3];
        val[u] = qf32 ? __float_as_uint(((const float*)qb)[o]) : (uint32_t)((const uint16_t*)qb)[o];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + 256 * u, r = e / HD, c = e % HD;
      if (qf32) ((uint32_t*)Qs)[r * QROWF + c] = val[u];
      else ((uint16_t*)Qs)[r * ROW + c] = (uint16_t)val[u];
    }
  }
  const int nchunks = (P.T + PF_CH - 1) / PF_CH;
  // live chunks: one warp per chunk, stopping at the first position above mask_skip
  for (int ch = warp; ch < nchunks; ch += 8) {
    const int64_t c0 = (int64_t)ch * PF_CH;
    bool any = false;
    if (FAST) {  // 16 float4 per mask row of the chunk (T is a multiple of 4)
      for (int e0 = 0; e0 < nrows * 16; e0 += 128) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = e0 + 32 * u + lane;
          const int64_t pos = c0 + 4 * (e & 15);
          if (e < nrows * 16 && pos < P.T) {
            const float4 m4 = P.mask_mode ? make_float4(mask_at(P, mb, moff_s[e >> 4], pos, qp0),
                                                        mask_at(P, mb, moff_s[e >> 4], pos + 1, qp0),
                                                        mask_at(P, mb, moff_s[e >> 4], pos + 2, qp0),
                                                        mask_at(P, mb, moff_s[e >> 4], pos + 3, qp0))
                                          : *(const float4*)(mf + moff_s[e >> 4] + pos);
            any |= fmaxf(fmaxf(m4.x, m4.y), fmaxf(m4.z, m4.w)) > P.mask_skip;
          }
        }
        if (__any_sync(0xffffffffu, any)) break;
      }
    } else {
      for (int e0 = 0; e0 < nrows * PF_CH; e0 += 128) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = e0 + 32 * u + lane;
          const int64_t pos = c0 + (e % PF_CH);
          if (e < nrows * PF_CH && pos < P.T && mask_at(P, mb, moff_s[e / PF_CH], pos, qp0) > P.mask_skip)
            any = true;
        }
        if (__any_sync(0xffffffffu, any)) break;
      }
    }
    if (__any_sync(0xffffffffu, any) && lane == 0) atomicOr(&live_s[ch >> 5], 1u << (ch & 31));
  }
  __syncthreads();
  auto next_live = [&](int from) {
    while (from < nchunks) {
      const unsigned w = live_s[from >> 5] >> (from & 31);
      if (w) return from + __ffs(w) - 1;
      from = (from | 31) + 1;
    }
    return nchunks;
  };
  constexpr int SEGS = HD / 8;
  // V rows of a chunk into the single V buffer (one cp.async group)
  auto stage_v = [&](int ch) {
    const int64_t c0 = (int64_t)ch * PF_CH;
    for (int q = threadIdx.x; q < PF_CH * SEGS; q += 256) {
      const int rr = q / SEGS, sg = q % SEGS;
      uint16_t* vd = Vb + (size_t)rr * ROW + sg * 8;
      if (c0 + rr < P.T) cp_async16(vd, vbase + (c0 + rr) * P.v.stride[2] + sg * 8);
      else *(uint4*)vd = make_uint4(0, 0, 0, 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // K rows and (FAST) the mask tile of a chunk into K buffer buf (one group)
  auto stage = [&](int ch, int buf) {
    const int64_t c0 = (int64_t)ch * PF_CH;
    for (int q = threadIdx.x; q < PF_CH * SEGS; q += 256) {
      const int rr = q / SEGS, sg = q % SEGS;
      uint16_t* kd = Kb + ((size_t)buf * PF_CH + rr) * ROW + sg * 8;
      if (c0 + rr < P.T) cp_async16(kd, kbase + (c0 + rr) * P.k.stride[2] + sg * 8);
      else *(uint4*)kd = make_uint4(0, 0, 0, 0);
    }
    if (FAST) {  // the chunk's mask tile; -inf past T and in rows past nrows
      for (int q = threadIdx.x; q < PF_ROWS * 16; q += 256) {
        const int r = q >> 4, sg = q & 15;
        const int64_t pos = c0 + 4 * sg;
        float* md = Ms + ((size_t)buf * PF_ROWS + r) * PF_MROW + 4 * sg;
        if (r < nrows && pos < P.T && P.mask_mode)
          *(float4*)md = make_float4(mask_at(P, mb, moff_s[r], pos, qp0), mask_at(P, mb, moff_s[r], pos + 1, qp0),
                                     mask_at(P, mb, moff_s[r], pos + 2, qp0), mask_at(P, mb, moff_s[r], pos + 3, qp0));
        else if (r < nrows && pos < P.T) cp_async16(md, mf + moff_s[r] + pos);
        else *(float4*)md = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // the closed-form chain (FAST): d1 rounding, multiply, its rounding
  const bool d1b = P.dt_d1 == KDT_BF16, mul = P.chain_kind == 1, mulb = P.chain_dt == KDT_BF16;
  const float cmul = P.chain_c, skip = P.mask_skip;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[NTO][4];
#pragma unroll
  for (int n = 0; n < NTO; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[n][i] = 0.f;
  const uint32_t kb_s = (uint32_t)__cvta_generic_to_shared(Kb), vb_s = (uint32_t)__cvta_generic_to_shared(Vb);
  const int rA = 16 * rg + g, rB = rA + 8;  // this thread's two rows
  // cp.async groups in commit order: K(ch) V(ch) K(nx) V(nx) ...; the K group of
  // a chunk is waited for before its scores, its V group before its P V
  int ch = next_live(0);
  if (ch < nchunks) {
    stage(ch, 0);
    stage_v(ch);
  }
  __syncthreads();  // Q in shared memory
  int buf = 0;
  while (ch < nchunks) {
    const int nx = next_live(ch + 1);
    if (nx < nchunks) {
      stage(nx, buf ^ 1);
      asm volatile("cp.async.wait_group 2;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    }
    __syncthreads();
    const int64_t c = (int64_t)ch * PF_CH;
    // scores of this warp's 16 rows over its half of the chunk: tiles
    // 4 dh .. 4 dh + 3 of 8 positions (the partner warp scores the other half)
    float sc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[n][i] = 0.f;
    const int mi = lane >> 3, ri = lane & 7;
#pragma unroll 2
    for (int kk = 0; kk < KSTEPS; ++kk) {
      // A fragments of the warp's rows (f32 queries: three exact bf16 parts)
      float qf[4][2];
      uint32_t a[4];
      if (qf32) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = (i & 1) ? rB : rA, col = 16 * kk + 2 * t + 8 * (i >> 1);
          const float2 v = *(const float2*)(Qs + (size_t)(row * QROWF + col) * 4);
          qf[i][0] = v.x;
          qf[i][1] = v.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = (i & 1) ? rB : rA, col = 16 * kk + 2 * t + 8 * (i >> 1);
          a[i] = *(const uint32_t*)(Qs + (size_t)(row * ROW + col) * 2);
        }
      }
      const int parts = qf32 ? 3 : 1;
      for (int part = 0; part < parts; ++part) {
        if (qf32)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            a[i] = pack_bf16(qf[i][0], qf[i][1]);
            qf[i][0] -= bf16_lo_f(a[i]);
            qf[i][1] -= bf16_hi_f(a[i]);
          }
#pragma unroll
        for (int n = 0; n < 4; n += 2) {
          uint32_t bf[4];
          ldsm_x4(kb_s + (uint32_t)((((size_t)buf * PF_CH + 8 * (4 * dh + n) + ri + 8 * (mi >> 1)) * ROW + 16 * kk + 8 * (mi & 1)) * 2), bf);
          mma_bf16(sc[n], a[0], a[1], a[2], a[3], bf[0], bf[1]);
          mma_bf16(sc[n + 1], a[0], a[1], a[2], a[3], bf[2], bf[3]);
        }
      }
    }
    // chain and mask (rows rA: elements 0, 1; rB: 2, 3), this half's row maxima
    float mxr[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = hr ? rB : rA;
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int tile = 4 * dh + n;
        if (FAST) {
          const float2 mk2 = *(const float2*)(Ms + ((size_t)buf * PF_ROWS + r) * PF_MROW + 8 * tile + 2 * t);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float mk = e ? mk2.y : mk2.x;
            float s = sc[n][2 * hr + e];
            if (d1b) s = bf16_round(s);
            if (mul) {
              s *= cmul;
              if (mulb) s = bf16_round(s);
            }
            const float v = mk > skip ? s + mk : -INFINITY;
            sc[n][2 * hr + e] = v;
            mx = fmaxf(mx, v);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int64_t j = c + 8 * tile + 2 * t + e;
            float v = -INFINITY;
            if (r < nrows && j < P.T) {
              const float mk = mask_at(P, mb, moff_s[r], j, qp0);
              if (mk > skip) v = rnd_dt(apply_chain(P, rnd_dt(sc[n][2 * hr + e], P.dt_d1)) + mk, P.dt_m);
            }
            sc[n][2 * hr + e] = v;
            mx = fmaxf(mx, v);
          }
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mxr[hr] = mx;
    }
    // the chunk's row maxima: this half's and the partner's, the same in both warps
    if (t == 0) {
      pm_s[dh][rA] = mxr[0];
      pm_s[dh][rB] = mxr[1];
    }
    pair_sync(rg);
    mxr[0] = fmaxf(mxr[0], pm_s[dh ^ 1][rA]);
    mxr[1] = fmaxf(mxr[1], pm_s[dh ^ 1][rB]);
    // online softmax: both warps apply the same maxima, each keeps the sum of its half
    float pv[4][4];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const float mnew = fmaxf(m[hr], mxr[hr]);
      float ps = 0.f;
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = sc[n][2 * hr + e];
          float p = 0.f;
          if (v != -INFINITY) p = FAST ? expf(v - mnew) : rnd_dt(expf(rnd_dt(v - mnew, P.dt_sub)), P.dt_exp);
          pv[n][2 * hr + e] = p;
          ps += p;
        }
      ps += __shfl_xor_sync(0xffffffffu, ps, 1);
      ps += __shfl_xor_sync(0xffffffffu, ps, 2);
      if (mnew != -INFINITY) {
        const float scl = m[hr] == -INFINITY ? 0.f : expf(m[hr] - mnew);
        l[hr] = l[hr] * scl + ps;
#pragma unroll
        for (int n = 0; n < NTO; ++n) {
          o[n][2 * hr] *= scl;
          o[n][2 * hr + 1] *= scl;
        }
        m[hr] = mnew;
      }
    }
    // P of this half (k-steps 2 dh, 2 dh + 1) as f32 in registers, published to
    // the partner through shared memory; both enter P V as the exact bf16
    // split hi + mid + lo (8 + 8 + 8 significand bits, the f32 value itself)
    float pr[2][8];
#pragma unroll
    for (int kl = 0; kl < 2; ++kl)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tile = 2 * kl + (i >> 1), hr = i & 1;
        pr[kl][2 * i] = pv[tile][2 * hr];
        pr[kl][2 * i + 1] = pv[tile][2 * hr + 1];
        pf_s[rg][dh][kl][2 * i][lane] = pr[kl][2 * i];
        pf_s[rg][dh][kl][2 * i + 1][lane] = pr[kl][2 * i + 1];
      }
    // this chunk's V rows (the barrier also publishes the P fragments)
    if (nx < nchunks) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // O[:, half] += P V: 4 k-steps of 16 positions, P as bf16 hi + mid + lo
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t ah[4], am[4], al[4];
      const int kl = ks & 1;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float p0, p1;
        if ((ks >> 1) == dh) {
          p0 = pr[kl][2 * i];
          p1 = pr[kl][2 * i + 1];
        } else {
          p0 = pf_s[rg][dh ^ 1][kl][2 * i][lane];
          p1 = pf_s[rg][dh ^ 1][kl][2 * i + 1][lane];
        }
        ah[i] = pack_bf16(p0, p1);
        const float r0 = p0 - bf16_lo_f(ah[i]), r1 = p1 - bf16_hi_f(ah[i]);
        am[i] = pack_bf16(r0, r1);
        al[i] = pack_bf16(r0 - bf16_lo_f(am[i]), r1 - bf16_hi_f(am[i]));
      }
#pragma unroll
      for (int n = 0; n < NTO; n += 2) {
        uint32_t bf[4];
        ldsm_x4_t(vb_s + (uint32_t)((((size_t)16 * ks + ri + 8 * (mi & 1)) * ROW + dh * (HD / 2) + 8 * n + 8 * (mi >> 1)) * 2), bf);
        mma_bf16(o[n], ah[0], ah[1], ah[2], ah[3], bf[0], bf[1]);
        mma_bf16(o[n + 1], ah[0], ah[1], ah[2], ah[3], bf[2], bf[3]);
        mma_bf16(o[n], am[0], am[1], am[2], am[3], bf[0], bf[1]);
        mma_bf16(o[n + 1], am[0], am[1], am[2], am[3], bf[2], bf[3]);
        mma_bf16(o[n], al[0], al[1], al[2], al[3], bf[0], bf[1]);
        mma_bf16(o[n + 1], al[0], al[1], al[2], al[3], bf[2], bf[3]);
      }
    }
    __syncthreads();  // this K buffer and the V buffer are restaged from here on
    if (nx < nchunks) stage_v(nx);
    ch = nx;
    buf ^= 1;
  }
  // out = O / l for this warp's rows and half of head_dim; l sums both halves
  if (t == 0) {
    pm_s[dh][rA] = l[0];
    pm_s[dh][rB] = l[1];
  }
  pair_sync(rg);
  l[0] += pm_s[dh ^ 1][rA];
  l[1] += pm_s[dh ^ 1][rB];
  char* ob = dres(P.out, argtab);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = hr ? rB : rA;
    if (r >= nrows) continue;
    const int qi = i0 + r / P.group, h = kh * P.group + r % P.group;
    const int64_t row = ((int64_t)b * P.nq + h) * P.Sq + qi;
#pragma unroll
    for (int n = 0; n < NTO; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int d = dh * (HD / 2) + 8 * n + 2 * t + e;
        const float v = l[hr] > 0.f ? o[n][2 * hr + e] / l[hr] : 0.f;
        if (P.out_dt == KDT_F32) ((float*)ob)[row * HD + d] = v;
        else ((__nv_bfloat16*)ob)[row * HD + d] = __float2bfloat16_rn(v);
      }
  }
}

// dynamic shared memory of the prefill kernel
int prefill_smem(const AttnParams& p, bool fast) {
  const int qbytes = p.q.dt == KDT_F32 ? PF_ROWS * (p.hd + 4) * 4 : PF_ROWS * (p.hd + 8) * 2;
  return 3 * PF_CH * (p.hd + 8) * 2 + (fast ? 2 * PF_ROWS * PF_MROW * 4 : 0) + qbytes;
}
constexpr int PF_SMEM_MAX = 227 * 1024 - 20 * 1024;  // the opt-in limit less the static shared memory

// the specialised form applies: f32 mask with 16-byte aligned rows, f32
// softmax arithmetic, a closed-form chain, and the mask tiles fit
bool prefill_fast(const AttnParams& p) {
  if (p.T % 4) return false;
  if (!p.mask_mode) {  // a computed mask has no rows to load
    if (p.mask.dt != KDT_F32 || p.mask.stride[3] != 1 || (p.mask.p.off % 16)) return false;
    for (int d = 0; d < 3; ++d)
      if (p.mask.stride[d] % 4) return false;
  }
  if (p.dt_m != KDT_F32 || p.dt_sub != KDT_F32 || p.dt_exp != KDT_F32) return false;
  if (!(p.dt_d1 == KDT_BF16 || p.dt_d1 == KDT_F32)) return false;
  if (!(p.chain_kind == 2 || (p.chain_kind == 1 && (p.chain_dt == KDT_BF16 || p.chain_dt == KDT_F32)))) return false;
  return prefill_smem(p, true) <= PF_SMEM_MAX;
}

template <int HD, bool FAST>
void launch_tc_prefill_t(const AttnParams& p, const uint64_t* argtab, cudaStream_t s) {
  ensure_smem_optin((const void*)attn_tc_prefill_kernel<HD, FAST>, PF_SMEM_MAX);
  const int qt = PF_ROWS / p.group;
  launch_k(attn_tc_prefill_kernel<HD, FAST>, dim3(1, (unsigned)((p.Sq + qt - 1) / qt), (unsigned)(p.B * p.nkv)),
           dim3(256), prefill_smem(p, FAST), s, 1, p, argtab);
}

template <int HD>
void launch_tc_prefill(const AttnParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (prefill_fast(p)) launch_tc_prefill_t<HD, true>(p, argtab, s);
  else launch_tc_prefill_t<HD, false>(p, argtab, s);
}

template <int HD>
void launch_tc(const AttnParams& p, const uint64_t* argtab, cudaStream_t s) {
  const int nbuf = (p.T + p.splits - 1) / p.splits > TC_CH ? 2 : 1;  // as the kernel decides
  const int dyn = nbuf * 2 * TC_CH * (HD + 8) * 2;
  ensure_smem_optin((const void*)attn_tc_kernel<HD>, 2 * 2 * TC_CH * (HD + 8) * 2);
  launch_k(attn_tc_kernel<HD>, dim3((unsigned)p.splits, 1, (unsigned)(p.B * p.nkv)), dim3(128), dyn, s, 1, p, argtab);
}

int dec_smem_bytes(const AttnParams& p, int nq) {
  const int64_t stage = 4LL * DEC_CH * p.hd + 8LL * nq * DEC_CH;    // K, V rows; mask and score rows
  const int64_t red = 4LL * (DEC_THREADS / 32) * nq * p.hd;         // the warps' contexts
  const int64_t merge = p.splits > 1 ? 4LL * p.splits * p.group * dec_part_stride(p.hd) : 0;  // every split's rows
  return (int)std::max(stage, std::max(red, merge));
}

int dec_nq(int group) { return group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : 8; }

template <int HD, int NQ>
void launch_dec_t(const AttnParams& p, const uint64_t* argtab, cudaStream_t s) {
  const int smem = dec_smem_bytes(p, NQ);
  ensure_smem_optin((const void*)attn_dec_kernel<HD, NQ>, smem);
  launch_k(attn_dec_kernel<HD, NQ>, dim3((unsigned)p.splits, (unsigned)(p.B * p.nkv)), dim3(DEC_THREADS), smem, s, 1,
           p, argtab);
}

template <int HD>
void launch_dec(const AttnParams& p, const uint64_t* argtab, cudaStream_t s) {
  switch (dec_nq(p.group)) {
    case 1: launch_dec_t<HD, 1>(p, argtab, s); return;
    case 2: launch_dec_t<HD, 2>(p, argtab, s); return;
    case 4: launch_dec_t<HD, 4>(p, argtab, s); return;
    default: launch_dec_t<HD, 8>(p, argtab, s); return;
  }
}

template <int HPL, int NQV>
void launch_smem(const AttnParams& p, const uint64_t* argtab, cudaStream_t s, dim3 grid) {
  constexpr int HD = HPL * 32;
  const int dyn = 2 * CH * (HD + 8) * 2;
  ensure_smem_optin((const void*)attn_smem_kernel<HPL, NQV>, dyn);
  launch_k(attn_smem_kernel<HPL, NQV>, dim3(grid), dim3(NW * 32), dyn, s, 1, p, argtab);
}

bool smem_ok(const AttnParams& p) {
  if (p.k_dt != KDT_BF16 || p.k.dt != KDT_BF16 || p.v.dt != KDT_BF16) return false;
  if ((p.k.p.off % 16) || (p.v.p.off % 16)) return false;
  for (int d = 0; d < 3; ++d)
    if ((p.k.stride[d] % 8) || (p.v.stride[d] % 8)) return false;
  return p.k.stride[3] == 1 && p.v.stride[3] == 1;
}

template <int HPL>
void launch_smem_nqv(const AttnParams& p, const uint64_t* argtab, cudaStream_t s, dim3 grid, int nqv) {
  if (nqv <= 1) launch_smem<HPL, 1>(p, argtab, s, grid);
  else if (nqv <= 2) launch_smem<HPL, 2>(p, argtab, s, grid);
  else if (nqv <= 4) launch_smem<HPL, 4>(p, argtab, s, grid);
  else launch_smem<HPL, 8>(p, argtab, s, grid);
}

template <typename KT, int HPL>
void launch_hpl(const AttnParams& p, const uint64_t* argtab, cudaStream_t s) {
  dim3 grid((unsigned)p.splits, (unsigned)((p.Sq + p.qtile - 1) / p.qtile), (unsigned)(p.B * p.nkv));
  int nqv = p.qtile * p.group;
  if constexpr (sizeof(KT) == 2) {
    // staging pays off where few CTAs each cover a long stretch of positions
    // (decode); prefill's many query tiles re-read K/V and keep direct loads
    if (smem_ok(p) && p.Sq <= p.qtile) {
      launch_smem_nqv<HPL>(p, argtab, s, grid, nqv);
      return;
    }
  }
  if (nqv <= 1) launch_k(attn_kernel<KT, HPL, 1>, dim3(grid), dim3(NW * 32), 0, s, 1, p, argtab);
  else if (nqv <= 2) launch_k(attn_kernel<KT, HPL, 2>, dim3(grid), dim3(NW * 32), 0, s, 1, p, argtab);
  else if (nqv <= 4) launch_k(attn_kernel<KT, HPL, 4>, dim3(grid), dim3(NW * 32), 0, s, 1, p, argtab);
  else launch_k(attn_kernel<KT, HPL, 8>, dim3(grid), dim3(NW * 32), 0, s, 1, p, argtab);
}

}  // namespace

void launch_attention(const AttnParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.use_tc == 3) {
    switch (p.hd) {
      case 32: launch_dec<32>(p, argtab, s); return;
      case 64: launch_dec<64>(p, argtab, s); return;
      case 128: launch_dec<128>(p, argtab, s); return;
      case 256: launch_dec<256>(p, argtab, s); return;
    }
    fail(E_INTERNAL, "staged decode attention: unsupported head_dim");
  }
  if (p.use_tc == 2) {
    switch (p.hd) {
      case 64: launch_tc_prefill<64>(p, argtab, s); return;
      case 128: launch_tc_prefill<128>(p, argtab, s); return;
      case 256: launch_tc_prefill<256>(p, argtab, s); return;
    }
    fail(E_INTERNAL, "tensor-core prefill attention: unsupported head_dim");
  }
  if (p.use_tc) {
    switch (p.hd) {
      case 64: launch_tc<64>(p, argtab, s); return;
      case 128: launch_tc<128>(p, argtab, s); return;
      case 256: launch_tc<256>(p, argtab, s); return;
    }
    fail(E_INTERNAL, "tensor-core attention: unsupported head_dim");
  }
  if (p.k_dt == KDT_BF16) {
    switch (p.hd) {
      case 32: launch_hpl<uint16_t, 1>(p, argtab, s); break;
      case 64: launch_hpl<uint16_t, 2>(p, argtab, s); break;
      case 128: launch_hpl<uint16_t, 4>(p, argtab, s); break;
      case 256: launch_hpl<uint16_t, 8>(p, argtab, s); break;
    }
  } else {
    switch (p.hd) {
      case 32: launch_hpl<float, 1>(p, argtab, s); break;
      case 64: launch_hpl<float, 2>(p, argtab, s); break;
      case 128: launch_hpl<float, 4>(p, argtab, s); break;
      case 256: launch_hpl<float, 8>(p, argtab, s); break;
    }
  }
}

bool attention_tc_prefill_ok(const AttnParams& p) {
  if (!(p.hd == 64 || p.hd == 128 || p.hd == 256) || !(p.q.dt == KDT_BF16 || p.q.dt == KDT_F32)) return false;
  if (!(p.group == 1 || p.group == 2 || p.group == 4 || p.group == 8)) return false;
  if (p.T > PF_LIVE_WORDS * 32 * PF_CH || prefill_smem(p, false) > PF_SMEM_MAX) return false;
  return smem_ok(p);
}

bool attention_dec_ok(const AttnParams& p) {
  if (!(p.hd == 32 || p.hd == 64 || p.hd == 128 || p.hd == 256) || p.Sq != 1 || p.group < 1 || p.group > 8) return false;
  if (!(p.q.dt == KDT_BF16 || p.q.dt == KDT_F32 || p.q.dt == KDT_F16)) return false;
  if (!(p.mask.dt == KDT_BF16 || p.mask.dt == KDT_F32 || p.mask.dt == KDT_F16)) return false;
  return smem_ok(p);
}

void plan_attention_dec(AttnParams& p, int sms) {
  (void)sms;  // a split per DEC_CH positions: the CTAs are short, several run per SM
  int64_t per = DEC_CH;
  if (const char* e = getenv("CLJXLA_B200_ATTN_SPLIT"))  // positions per split (measurement sweeps)
    if (atoi(e) >= 16) per = atoi(e);
  // at most ATTN_MERGE_MAX_SPLITS splits, and the merging CTA's copy of every
  // split's partial rows within 200 KB of shared memory
  const int64_t cap = std::max<int64_t>(1, std::min<int64_t>(ATTN_MERGE_MAX_SPLITS,
                                                             200 * 1024 / (4LL * p.group * dec_part_stride(p.hd))));
  while ((p.T + per - 1) / per > cap) per += DEC_CH;
  p.splits = (int32_t)((p.T + per - 1) / per);
  p.dec_per_split = (int32_t)per;
  p.dec_chunk = DEC_CH;
}

int64_t attention_part_bytes(const AttnParams& p) {
  const int64_t rows = (int64_t)p.B * p.nq * p.Sq;
  return (int64_t)p.splits * rows * (p.use_tc == 3 ? dec_part_stride(p.hd) : p.hd + 2) * 4;
}

bool attention_tc_ok(const AttnParams& p) {
  if (!(p.hd == 64 || p.hd == 128 || p.hd == 256) || !(p.q.dt == KDT_BF16 || p.q.dt == KDT_F32)) return false;
  if (p.Sq > p.qtile || p.Sq * p.group > 8 || p.Sq < 1) return false;
  return smem_ok(p);
}

void launch_attention_combine(const AttnParams& p, const uint64_t* argtab, cudaStream_t s) {
  int64_t rows = (int64_t)p.B * p.nq * p.Sq;
  int g = (int)(rows < 65535 ? rows : 65535);
  launch_k(attn_combine_kernel, dim3(g), dim3(p.hd < 256 ? p.hd : 256), 0, s, 1, p, argtab);
}

void verify_attention(const Launch& l, const RegionFn& region) {
  const AttnParams& p = *(const AttnParams*)l.blob.data();
  auto vext = [&](const TView& v, const char* what) {
    int64_t hi = 0;
    for (int i = 0; i < v.rank; ++i) {
      if (v.shape[i] == 0) return;
      if (v.stride[i] < 0) fail(E_INTERNAL, "negative stride in attention view");
      hi += (v.shape[i] - 1) * v.stride[i];
    }
    region(v.p, (hi + 1) * (int64_t)dt_size((DT)v.dt), what);
  };
  vext(p.q, "q");
  vext(p.k, "k");
  vext(p.v, "v");
  if (p.mask_mode) {
    if (p.has_mask_pos) region(p.mask_pos, 4, "mask position");
    if (p.mask.stride[0] || p.mask.stride[1] || p.mask.stride[2] != 1 || p.mask.stride[3] || p.mask_mode != 1)
      fail(E_INTERNAL, "computed attention mask with a bad view");
  } else {
    vext(p.mask, "mask");
  }
  int64_t rows = (int64_t)p.B * p.nq * p.Sq;
  region(p.out, rows * p.hd * (int64_t)dt_size((DT)p.out_dt), "out");
  if (p.splits > 1) region(p.part, attention_part_bytes(p), "partials");
  if (p.splits > 1 && p.use_counters) {
    region(p.counters, 4LL * p.B * p.nkv * ((p.Sq + p.qtile - 1) / p.qtile), "arrival counters");
    if (p.splits > ATTN_MERGE_MAX_SPLITS || p.qtile * p.group > 8) fail(E_INTERNAL, "attention merge too wide");
  }
  if (p.use_tc == 1 && !attention_tc_ok(p)) fail(E_INTERNAL, "tensor-core attention on unsupported views");
  if (p.use_tc == 3) {
    if (!attention_dec_ok(p)) fail(E_INTERNAL, "staged decode attention on unsupported views");
    if (p.dec_per_split < 1 || (int64_t)p.splits * p.dec_per_split < p.T ||
        (int64_t)(p.splits - 1) * p.dec_per_split >= p.T || p.dec_chunk != DEC_CH ||
        dec_smem_bytes(p, dec_nq(p.group)) > 220 * 1024 || (p.splits > 1 && !p.use_counters) ||
        (p.part.off % 16))
      fail(E_INTERNAL, "staged decode attention: bad split / chunk sizes");
    if (p.has_status) region(p.status, 4, "status word");
    if (p.nhint < 0 || p.nhint > ATTN_MAX_HINTS) fail(E_INTERNAL, "staged decode attention: bad hint list");
    for (int h = 0; h < p.nhint; ++h) {
      if (p.hint_bytes[h] % 16 || p.hint[h].off % 16 || p.hint_bytes[h] <= 0)
        fail(E_INTERNAL, "staged decode attention: unaligned hint");
      region(p.hint[h], p.hint_bytes[h], "prefetched weights");
    }
  }
  if (p.dec_live_splits && (p.use_tc != 3 || p.mask_mode != 1))
    fail(E_INTERNAL, "live-position splits without a computed mask");
  if (p.use_tc == 2 && (!attention_tc_prefill_ok(p) || p.splits != 1))
    fail(E_INTERNAL, "tensor-core prefill attention on unsupported views");
  if (p.q.shape[0] != p.B || p.q.shape[1] != p.nq || p.q.shape[2] != p.Sq || p.q.shape[3] != p.hd ||
      p.k.shape[1] != p.nkv || p.k.shape[2] != p.T || p.k.shape[3] != p.hd || p.v.shape[2] != p.T ||
      p.mask.shape[3] != p.T || p.k.stride[3] != 1 || p.v.stride[3] != 1 || p.nq != p.nkv * p.group)
    fail(E_INTERNAL, "attention view shapes inconsistent");
  if (p.nchain > 12 || p.chain_out >= 16) fail(E_INTERNAL, "attention chain too long");
  for (int i = 0; i < p.nchain; ++i)
    if (p.chain[i].dst >= 16 || p.chain[i].a >= 16 || p.chain[i].b >= 16) fail(E_INTERNAL, "attention chain register");
}

}  // namespace cljxla
