// Elementwise register-program step shared by the fused elementwise and
// fused row kernels (device code, included by both translation units).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kernels.h"

namespace cljxla {
namespace {

__device__ __forceinline__ uint32_t ld_elem(const char* base, int64_t i, int dt) {
  switch (dt) {
    case KDT_F32: return __float_as_uint(((const float*)base)[i]);
    case KDT_BF16: return (uint32_t)((const uint16_t*)base)[i] << 16;
    case KDT_F16: return __float_as_uint(__half2float(((const __half*)base)[i]));
    case KDT_I32: case KDT_U32: return (uint32_t)((const int32_t*)base)[i];
    case KDT_I8: return (uint32_t)(int32_t)((const int8_t*)base)[i];
    case KDT_U8: return (uint32_t)((const uint8_t*)base)[i];
    case KDT_I16: return (uint32_t)(int32_t)((const int16_t*)base)[i];
    case KDT_I1: return ((const uint8_t*)base)[i] ? 1u : 0u;
    case KDT_I64: return (uint32_t)(int32_t)((const int64_t*)base)[i];
    case KDT_F64: return __float_as_uint((float)((const double*)base)[i]);
  }
  return 0;
}

__device__ __forceinline__ void st_elem(char* base, int64_t i, int dt, uint32_t v) {
  switch (dt) {
    case KDT_F32: ((float*)base)[i] = __uint_as_float(v); break;
    case KDT_BF16: {
      __nv_bfloat16 b = __float2bfloat16_rn(__uint_as_float(v));
      ((__nv_bfloat16*)base)[i] = b;
      break;
    }
    case KDT_F16: ((__half*)base)[i] = __float2half_rn(__uint_as_float(v)); break;
    case KDT_I32: case KDT_U32: ((int32_t*)base)[i] = (int32_t)v; break;
    case KDT_I8: ((int8_t*)base)[i] = (int8_t)(int32_t)v; break;
    case KDT_U8: ((uint8_t*)base)[i] = (uint8_t)v; break;
    case KDT_I16: ((int16_t*)base)[i] = (int16_t)(int32_t)v; break;
    case KDT_I1: ((uint8_t*)base)[i] = v ? 1 : 0; break;
    case KDT_I64: ((int64_t*)base)[i] = (int64_t)(int32_t)v; break;
    case KDT_F64: ((double*)base)[i] = (double)__uint_as_float(v); break;
  }
}

__device__ __forceinline__ bool is_float_dt(int dt) {
  return dt == KDT_F32 || dt == KDT_BF16 || dt == KDT_F16 || dt == KDT_F64;
}

// round an f32 value to the value set of a floating element type
__device__ __forceinline__ float rnd(float v, int dt) {
  if (dt == KDT_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == KDT_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ uint32_t fbits(float v, int dt) { return __float_as_uint(rnd(v, dt)); }

__device__ uint32_t ew_convert(uint32_t v, int from, int to) {
  bool ff = is_float_dt(from), tf = is_float_dt(to);
  if (to == KDT_I1) return ff ? (__uint_as_float(v) != 0.0f) : (v != 0);
  if (ff && tf) return fbits(__uint_as_float(v), to);
  if (!ff && tf) {
    float f = (from == KDT_U32) ? (float)v : (float)(int32_t)v;
    return fbits(f, to);
  }
  if (ff && !tf) {
    float f = __uint_as_float(v);
    int32_t r;
    if (f != f) r = 0;
    else if (f >= 2147483647.0f) r = 2147483647;
    else if (f <= -2147483648.0f) r = (int32_t)0x80000000;
    else r = (int32_t)f;  // truncation toward zero
    if (to == KDT_I8) r = (int8_t)r;
    else if (to == KDT_U8) r = (uint8_t)r;
    else if (to == KDT_I16) r = (int16_t)r;
    return (uint32_t)r;
  }
  int32_t r = (int32_t)v;
  if (to == KDT_I8) r = (int8_t)r;
  else if (to == KDT_U8) r = (uint8_t)r;
  else if (to == KDT_I16) r = (int16_t)r;
  return (uint32_t)r;
}


// one instruction; idx = loop multi-index, R = register file
__device__ __forceinline__ void ew_step(const EwInstr& I, uint32_t* R, const int64_t* idx, int rank,
                                        const EwIn* ins, const uint64_t* __restrict__ argtab) {
      uint32_t r = 0;
      const int dt = I.dt;
      const bool fl = is_float_dt(dt);
      switch (I.op) {
        case EW_LOAD: {
          const EwIn& in = ins[I.aux];
          if (in.sel_dim >= 0) {
            const int64_t k = idx[in.sel_dim];
            if (k < in.sel_lo || k >= in.sel_hi) {  // another concatenate operand covers this index
              r = R[I.b];
              break;
            }
            int64_t off = (k - in.sel_lo) * in.stride[in.sel_dim];
            for (int d = 0; d < rank; ++d)
              if (d != in.sel_dim) off += idx[d] * in.stride[d];
            r = ld_elem(dres(in.p, argtab), off, in.dt);
            break;
          }
          int64_t off = 0;
          for (int d = 0; d < rank; ++d) off += idx[d] * in.stride[d];
          r = ld_elem(dres(in.p, argtab), off, in.dt);
          break;
        }
        case EW_IMM: r = fl ? __float_as_uint(I.fimm) : (uint32_t)I.iimm; break;
        case EW_IOTA: r = fl ? fbits((float)idx[I.aux], dt) : (uint32_t)idx[I.aux]; break;
        case EW_ADD: case EW_SUB: case EW_MUL: case EW_DIV: case EW_MAX: case EW_MIN: {
          uint32_t a = R[I.a], b = R[I.b];
          if (fl) {
            float x = __uint_as_float(a), y = __uint_as_float(b), z;
            switch (I.op) {
              case EW_ADD: z = x + y; break;
              case EW_SUB: z = x - y; break;
              case EW_MUL: z = x * y; break;
              case EW_DIV: z = x / y; break;
              case EW_MAX: z = (x != x || y != y) ? __int_as_float(0x7fc00000) : fmaxf(x, y); break;
              default: z = (x != x || y != y) ? __int_as_float(0x7fc00000) : fminf(x, y); break;
            }
            r = fbits(z, dt);
          } else {
            int32_t x = (int32_t)a, y = (int32_t)b, z;
            switch (I.op) {
              case EW_ADD: z = x + y; break;
              case EW_SUB: z = x - y; break;
              case EW_MUL: z = x * y; break;
              case EW_DIV: z = y == 0 ? -1 : x / y; break;
              case EW_MAX: z = x > y ? x : y; break;
              default: z = x < y ? x : y; break;
            }
            if (dt == KDT_I1) z = z ? 1 : 0;
            r = (uint32_t)z;
          }
          break;
        }
        case EW_EXP: case EW_TANH: case EW_SQRT: case EW_RSQRT: case EW_SIN: case EW_COS:
        case EW_LOGISTIC: case EW_NEG: case EW_ABS: {
          if (fl) {
            float x = __uint_as_float(R[I.a]), z;
            switch (I.op) {
              case EW_EXP: z = expf(x); break;
              case EW_TANH: z = tanhf(x); break;
              case EW_SQRT: z = sqrtf(x); break;
              case EW_RSQRT: z = 1.0f / sqrtf(x); break;
              case EW_SIN: z = sinf(x); break;
              case EW_COS: z = cosf(x); break;
              case EW_LOGISTIC: z = 1.0f / (1.0f + expf(-x)); break;
              case EW_NEG: z = -x; break;
              default: z = fabsf(x); break;
            }
            r = fbits(z, dt);
          } else {
            int32_t x = (int32_t)R[I.a];
            r = (uint32_t)(I.op == EW_NEG ? -x : (I.op == EW_ABS ? (x < 0 ? -x : x) : x));
          }
          break;
        }
        case EW_CONVERT: r = ew_convert(R[I.a], I.aux, dt); break;
        case EW_CMP: {
          uint32_t a = R[I.a], b = R[I.b];
          bool c;
          if (is_float_dt(I.aux2)) {
            float x = __uint_as_float(a), y = __uint_as_float(b);
            switch (I.aux) {
              case 0: c = x == y; break;
              case 1: c = x != y; break;
              case 2: c = x >= y; break;
              case 3: c = x > y; break;
              case 4: c = x <= y; break;
              default: c = x < y; break;
            }
          } else {
            int32_t x = (int32_t)a, y = (int32_t)b;
            switch (I.aux) {
              case 0: c = x == y; break;
              case 1: c = x != y; break;
              case 2: c = x >= y; break;
              case 3: c = x > y; break;
              case 4: c = x <= y; break;
              default: c = x < y; break;
            }
          }
          r = c ? 1u : 0u;
          break;
        }
        case EW_SELECT: r = R[I.a] ? R[I.b] : R[I.c]; break;
      }

      R[I.dst] = r;
}

}  // namespace
}  // namespace cljxla
