// Generic strided batched GEMM for dot_general: C[b][m][n] = sum_k A[b][m][k] B[b][k][n]
// with f32 / bf16 / f16 operands of any mix, exact f32 FFMA accumulation and
// the result rounded to the printed result type.  This is the correctness path
// for contractions the specialised kernels (decode GEMV, tcgen05 GEMM, fused
// attention) do not claim; it also keeps f32 graphs (GPT-2) at f32 precision.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "kernels.h"

namespace cljxla {
namespace {

__device__ __forceinline__ float ldf(const char* base, int64_t i, int dt) {
  if (dt == KDT_F32) return ((const float*)base)[i];
  if (dt == KDT_BF16) return __uint_as_float((uint32_t)((const uint16_t*)base)[i] << 16);
  return __half2float(((const __half*)base)[i]);
}

__device__ __forceinline__ void stf(char* base, int64_t i, int dt, float v) {
  if (dt == KDT_F32) ((float*)base)[i] = v;
  else if (dt == KDT_BF16) ((__nv_bfloat16*)base)[i] = __float2bfloat16_rn(v);
  else ((__half*)base)[i] = __float2half_rn(v);
}

constexpr int TM = 64, TN = 64, TK = 16;

__global__ void __launch_bounds__(256) gemm_generic_kernel(const __grid_constant__ GemmParams P,
                                                           const uint64_t* __restrict__ argtab) {
  pdl_enter();
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int64_t bz = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * TM, n0 = (int64_t)blockIdx.x * TN;
  const char* A = dres(P.a, argtab);
  const char* B = dres(P.b, argtab);
  char* C = dres(P.c, argtab);
  const int64_t aoff = bz * P.a_sb, boff = bz * P.b_sb;
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  float acc[4][4] = {};
  const bool a_k_fast = P.a_sk == 1;
  const bool b_n_fast = P.b_sn == 1;
  for (int64_t k0 = 0; k0 < P.K; k0 += TK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int e = tid + i * 256;  // 0..1023 over a 64x16 tile
      int mm, kk;
      if (a_k_fast) { mm = e / TK; kk = e % TK; } else { mm = e % TM; kk = e / TM; }
      int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < P.M && gk < P.K) ? ldf(A, aoff + gm * P.a_sm + gk * P.a_sk, P.a_dt) : 0.0f;
      int nn, kb;
      if (b_n_fast) { nn = e % TN; kb = e / TN; } else { nn = e / TK; kb = e % TK; }
      int64_t gn = n0 + nn, gkb = k0 + kb;
      Bs[kb][nn] = (gn < P.N && gkb < P.K) ? ldf(B, boff + gkb * P.b_sk + gn * P.b_sn, P.b_dt) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t gm = m0 + ty * 4 + i;
    if (gm >= P.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t gn = n0 + tx * 4 + j;
      if (gn < P.N) stf(C, bz * P.c_sb + gm * P.N + gn, P.c_dt, acc[i][j]);
    }
  }
}

// ---------------------------------------------------------------------------
// Few-row f32 products (GPT-2 decode: x[M <= 8, K] against f32 weights).  The
// tiled kernel above gives each 64 x 64 tile to one CTA, which for one row of
// x leaves most SMs idle and reads each weight once per 64 rows of x; these
// stream the weights once with 16-byte loads instead, f32 FFMA throughout.
//
// NN: W[K, N] with N contiguous (the [in, out] Conv1D weights of GPT-2,
// gpt2.clj:27-31).  A CTA owns 4 CG columns; its 256 threads are CG column
// groups (float4) x 256 / CG K lanes, each accumulating its columns over the
// rows k = lane, lane + KL, ...; the K lanes are summed through shared memory
// in lane order.
template <int CG, int MT>
__global__ void __launch_bounds__(256) gemv_f32_nn_kernel(const __grid_constant__ GemmParams P,
                                                          const uint64_t* __restrict__ argtab) {
  constexpr int KL = 256 / CG;
  __shared__ __align__(16) float red[KL][MT][4 * CG];
  pdl_enter();
  const float* X = (const float*)dres(P.a, argtab);
  const float* W = (const float*)dres(P.b, argtab);
  float* C = (float*)dres(P.c, argtab);
  const int cg = threadIdx.x % CG, kl = threadIdx.x / CG;
  const int64_t col = ((int64_t)blockIdx.x * CG + cg) * 4;
  const bool on = col < P.N;  // N % 4 == 0: the whole float4 is in range
  float4 acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (on) {
    int64_t k = kl;
    for (; k + 3 * KL < P.K; k += 4 * KL) {  // four rows in flight
      float4 w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) w[u] = __ldg((const float4*)(W + (k + u * KL) * P.b_sk + col));
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m >= P.M) break;
          const float xv = __ldg(X + m * P.a_sm + k + u * KL);
          acc[m].x = fmaf(xv, w[u].x, acc[m].x);
          acc[m].y = fmaf(xv, w[u].y, acc[m].y);
          acc[m].z = fmaf(xv, w[u].z, acc[m].z);
          acc[m].w = fmaf(xv, w[u].w, acc[m].w);
        }
    }
    for (; k < P.K; k += KL) {
      const float4 w = __ldg((const float4*)(W + k * P.b_sk + col));
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m >= P.M) break;
        const float xv = __ldg(X + m * P.a_sm + k);
        acc[m].x = fmaf(xv, w.x, acc[m].x);
        acc[m].y = fmaf(xv, w.y, acc[m].y);
        acc[m].z = fmaf(xv, w.z, acc[m].z);
        acc[m].w = fmaf(xv, w.w, acc[m].w);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) *(float4*)&red[kl][m][cg * 4] = acc[m];
  __syncthreads();
  for (int e = threadIdx.x; e < MT * 4 * CG; e += 256) {
    const int m = e / (4 * CG), c = e % (4 * CG);
    const int64_t gc = (int64_t)blockIdx.x * CG * 4 + c;
    if (m >= P.M || gc >= P.N) continue;
    float t = 0.f;
    for (int q = 0; q < KL; ++q) t += red[q][m][c];
    C[m * P.N + gc] = t;
  }
}

// NT: W[N, K] with K contiguous (GPT-2's LM head, transpose(wte)): a warp per
// row of W, 16-byte loads along K, x rows through the read-only cache.
template <int MT>
__global__ void __launch_bounds__(256) gemv_f32_nt_kernel(const __grid_constant__ GemmParams P,
                                                          const uint64_t* __restrict__ argtab) {
  pdl_enter();
  const float* X = (const float*)dres(P.a, argtab);
  const float* W = (const float*)dres(P.b, argtab);
  float* C = (float*)dres(P.c, argtab);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t K4 = P.K / 4;
  for (int64_t n = (int64_t)blockIdx.x * 8 + warp; n < P.N; n += (int64_t)gridDim.x * 8) {
    const float4* wr = (const float4*)(W + n * P.b_sn);
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    for (int64_t k4 = lane; k4 < K4; k4 += 32) {
      const float4 w = __ldg(wr + k4);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m >= P.M) break;
        const float4 xv = __ldg((const float4*)(X + m * P.a_sm) + k4);
        acc[m] = fmaf(xv.x, w.x, fmaf(xv.y, w.y, fmaf(xv.z, w.z, fmaf(xv.w, w.w, acc[m]))));
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    if (lane == 0)
      for (int m = 0; m < MT && m < P.M; ++m) C[m * P.N + n] = acc[m];
  }
}

template <int MT>
void launch_f32_nn(const GemmParams& p, const uint64_t* argtab, cudaStream_t s) {
  // the widest column group that still gives about 96 CTAs
  if (p.N / 32 >= 96) launch_k(gemv_f32_nn_kernel<8, MT>, dim3((unsigned)((p.N + 31) / 32)), dim3(256), 0, s, 1, p, argtab);
  else if (p.N / 16 >= 96) launch_k(gemv_f32_nn_kernel<4, MT>, dim3((unsigned)((p.N + 15) / 16)), dim3(256), 0, s, 1, p, argtab);
  else launch_k(gemv_f32_nn_kernel<2, MT>, dim3((unsigned)((p.N + 7) / 8)), dim3(256), 0, s, 1, p, argtab);
}

}  // namespace

bool gemv_f32_ok(const GemmParams& p, bool* nn) {
  if (p.batch != 1 || p.M < 1 || p.M > 8 || p.K < 1 || p.N < 1) return false;
  if (p.a_dt != KDT_F32 || p.b_dt != KDT_F32 || p.c_dt != KDT_F32 || p.a_sk != 1) return false;
  if (p.b_sn == 1 && p.N % 4 == 0 && p.b_sk % 4 == 0 && p.b_sk >= p.N && p.b.off % 16 == 0) {
    *nn = true;
    return true;
  }
  if (p.b_sk == 1 && p.K % 4 == 0 && p.b_sn % 4 == 0 && p.b_sn >= p.K && p.b.off % 16 == 0 && p.a.off % 16 == 0 &&
      (p.M == 1 || p.a_sm % 4 == 0)) {
    *nn = false;
    return true;
  }
  return false;
}

void launch_gemm(const GemmParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.M == 0 || p.N == 0 || p.batch == 0) return;
  bool nn = false;
  if (gemv_f32_ok(p, &nn)) {
    if (nn) {
      if (p.M == 1) launch_f32_nn<1>(p, argtab, s);
      else launch_f32_nn<8>(p, argtab, s);
    } else {
      const int64_t blocks = std::min<int64_t>((p.N + 7) / 8, 148 * 8);
      if (p.M == 1) launch_k(gemv_f32_nt_kernel<1>, dim3((unsigned)blocks), dim3(256), 0, s, 1, p, argtab);
      else launch_k(gemv_f32_nt_kernel<8>, dim3((unsigned)blocks), dim3(256), 0, s, 1, p, argtab);
    }
    return;
  }
  dim3 grid((unsigned)((p.N + TN - 1) / TN), (unsigned)((p.M + TM - 1) / TM), (unsigned)p.batch);
  launch_k(gemm_generic_kernel, dim3(grid), dim3(256), 0, s, 1, p, argtab);
}

}  // namespace cljxla
