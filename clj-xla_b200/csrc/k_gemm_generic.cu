// Generic strided batched GEMM for dot_general: C[b][m][n] = sum_k A[b][m][k] B[b][k][n]
// with f32 / bf16 / f16 operands of any mix, exact f32 FFMA accumulation and
// the result rounded to the printed result type.  This is the correctness path
// for contractions the specialised kernels (decode GEMV, tcgen05 GEMM, fused
// attention) do not claim; it also keeps f32 graphs (GPT-2) at f32 precision.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

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

}  // namespace

void launch_gemm(const GemmParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.M == 0 || p.N == 0 || p.batch == 0) return;
  dim3 grid((unsigned)((p.N + TN - 1) / TN), (unsigned)((p.M + TM - 1) / TM), (unsigned)p.batch);
  launch_k(gemm_generic_kernel, dim3(grid), dim3(256), 0, s, 1, p, argtab);
}

}  // namespace cljxla
