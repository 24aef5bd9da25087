// Generic kernels: every printed op the fused fast paths do not claim runs
// here on the GPU (there is no CPU fallback).  Fused elementwise regions run
// through a small register-program interpreter; reductions, strided copies
// (view materialisation, concatenate), gather and dynamic_update_slice have
// their own kernels.  All read operands through strided views so reshape /
// transpose / broadcast_in_dim / slice never copy unless a consumer needs a
// dense layout.
#include <cuda_bf16.h>
#include "ew_exec.cuh"

#include "kernels.h"

namespace cljxla {

namespace {

__global__ void __launch_bounds__(256) ew_kernel(const __grid_constant__ EwParams P,
                                                 const uint64_t* __restrict__ argtab) {
  pdl_enter();
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = tid; e < P.n; e += nthreads) {
    int64_t idx[CLJXLA_MAXR];
    if (P.rank == 1) {
      idx[0] = e;
    } else {
      int64_t rem = e;
      for (int d = P.rank - 1; d > 0; --d) {
        int64_t dim = P.dims[d];
        idx[d] = rem % dim;
        rem /= dim;
      }
      idx[0] = rem;
    }
    uint32_t R[EW_NREG];
    for (int pc = 0; pc < P.ncode; ++pc) {
      ew_step(P.code[pc], R, idx, P.rank, P.in, argtab);
    }
    for (int o = 0; o < P.nout; ++o) st_elem(dres(P.out[o].p, argtab), e, P.out[o].dt, R[P.out[o].reg]);
  }
}

__device__ __forceinline__ int64_t view_off(const TView& v, int64_t e) {
  int64_t off = 0;
  for (int d = v.rank - 1; d >= 0; --d) {
    int64_t dim = v.shape[d];
    off += (e % dim) * v.stride[d];
    e /= dim;
  }
  return off;
}

// byte copy between dense buffers: 16-byte vectors when both ends are aligned
__global__ void copy_bytes_kernel(DPtr srcp, DPtr dstp, int64_t bytes, int vec, const uint64_t* __restrict__ argtab) {
  pdl_enter();
  const char* src = dres(srcp, argtab);
  char* dst = dres(dstp, argtab);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, nt = (int64_t)gridDim.x * blockDim.x;
  if (vec == 16) {
    const int64_t n = bytes / 16;
    for (int64_t i = tid; i < n; i += nt) ((uint4*)dst)[i] = __ldcs(((const uint4*)src) + i);
  } else if (vec == 4) {
    const int64_t n = bytes / 4;
    for (int64_t i = tid; i < n; i += nt) ((uint32_t*)dst)[i] = ((const uint32_t*)src)[i];
  } else {
    for (int64_t i = tid; i < bytes; i += nt) dst[i] = src[i];
  }
}

__global__ void copy_kernel(const __grid_constant__ CopyParams P, const uint64_t* __restrict__ argtab) {
  pdl_enter();
  const char* src = dres(P.src.p, argtab);
  char* dst = dres(P.dst.p, argtab);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < P.n; e += (int64_t)gridDim.x * blockDim.x) {
    uint32_t v = ld_elem(src, view_off(P.src, e), P.src.dt);
    if (P.src.dt != P.dst.dt) v = ew_convert(v, P.src.dt, P.dst.dt);
    st_elem(dst, view_off(P.dst, e), P.dst.dt, v);
  }
}

template <int BLOCK>
__global__ void __launch_bounds__(BLOCK) reduce_kernel(const __grid_constant__ ReduceParams P,
                                                       const uint64_t* __restrict__ argtab) {
  pdl_enter();
  const char* src = dres(P.in.p, argtab);
  char* dst = dres(P.out, argtab);
  const bool fl = is_float_dt(P.in.dt);
  __shared__ float sf[BLOCK / 32];
  __shared__ int si[BLOCK / 32];
  for (int64_t o = blockIdx.x; o < P.n_out; o += gridDim.x) {
    int64_t base = 0, rem = o;
    for (int d = P.nkeep - 1; d >= 0; --d) {
      base += (rem % P.keep_shape[d]) * P.keep_stride[d];
      rem /= P.keep_shape[d];
    }
    float accf = P.kind == 0 ? 0.0f : -INFINITY;
    int32_t acci = P.kind == 0 ? 0 : (int32_t)0x80000000;
    for (int64_t r = threadIdx.x; r < P.n_red; r += BLOCK) {
      int64_t off = base;
      if (P.nred == 1) {
        off += r * P.red_stride[0];
      } else {
        int64_t rr = r;
        for (int d = P.nred - 1; d >= 0; --d) {
          off += (rr % P.red_shape[d]) * P.red_stride[d];
          rr /= P.red_shape[d];
        }
      }
      uint32_t v = ld_elem(src, off, P.in.dt);
      if (fl) {
        float x = __uint_as_float(v);
        accf = P.kind == 0 ? accf + x : fmaxf(accf, x);
      } else {
        int32_t x = (int32_t)v;
        acci = P.kind == 0 ? acci + x : max(acci, x);
      }
    }
    for (int sh = 16; sh > 0; sh >>= 1) {
      float of = __shfl_xor_sync(0xffffffffu, accf, sh);
      int32_t oi = __shfl_xor_sync(0xffffffffu, acci, sh);
      accf = P.kind == 0 ? accf + of : fmaxf(accf, of);
      acci = P.kind == 0 ? acci + oi : max(acci, oi);
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { sf[w] = accf; si[w] = acci; }
    __syncthreads();
    if (threadIdx.x == 0) {
      float tf = P.kind == 0 ? 0.0f : -INFINITY;
      int32_t ti = P.kind == 0 ? 0 : (int32_t)0x80000000;
      for (int k = 0; k < BLOCK / 32; ++k) {
        tf = P.kind == 0 ? tf + sf[k] : fmaxf(tf, sf[k]);
        ti = P.kind == 0 ? ti + si[k] : max(ti, si[k]);
      }
      uint32_t res;
      if (fl) {
        tf = P.kind == 0 ? tf + P.init : fmaxf(tf, P.init);
        res = fbits(tf, P.out_dt);
      } else {
        int32_t iv = (int32_t)P.init;
        ti = P.kind == 0 ? ti + iv : max(ti, iv);
        res = (uint32_t)ti;
      }
      st_elem(dst, o, P.out_dt, res);
    }
    __syncthreads();
  }
}

__global__ void gather_kernel(const __grid_constant__ GatherParams P, const uint64_t* __restrict__ argtab) {
  pdl_enter();
  const char* table = dres(P.table, argtab);
  const char* idxb = dres(P.idx.p, argtab);
  char* out = dres(P.out, argtab);
  const int64_t esz = P.table_dt == KDT_F32 ? 4 : 2;
  for (int64_t r = blockIdx.x; r < P.n_rows; r += gridDim.x) {
    int64_t row = (int32_t)ld_elem(idxb, view_off(P.idx, r), P.idx_dt);
    row = row < 0 ? 0 : (row >= P.rows_table ? P.rows_table - 1 : row);  // clamp (StableHLO gather)
    const char* src = table + row * P.table_row_stride * esz;
    char* dst = out + r * P.row_len * esz;
    const int64_t bytes = P.row_len * esz;
    if ((bytes & 15) == 0 && (((uintptr_t)src | (uintptr_t)dst) & 15) == 0) {
      for (int64_t b = threadIdx.x * 16; b < bytes; b += blockDim.x * 16)
        *(uint4*)(dst + b) = *(const uint4*)(src + b);
    } else {
      for (int64_t b = threadIdx.x; b < bytes; b += blockDim.x) dst[b] = src[b];
    }
  }
}

__device__ __forceinline__ int64_t dus_start(const DusParams& P, int d, const uint64_t* argtab) {
  int64_t s = P.start_imm[d];
  if (P.start_is_ptr[d]) s = (int32_t)ld_elem(dres(P.start_ptr[d], argtab), 0, P.start_dt[d]);
  int64_t hi = P.out_shape[d] - P.upd_shape[d];
  return s < 0 ? 0 : (s > hi ? hi : s);  // clamp so the update fits (StableHLO semantics)
}

__global__ void dus_kernel(const __grid_constant__ DusParams P, const uint64_t* __restrict__ argtab) {
  pdl_enter();
  int64_t st[CLJXLA_MAXR];
  for (int d = 0; d < P.rank; ++d) st[d] = dus_start(P, d, argtab);
  const char* opnd = dres(P.operand.p, argtab);
  const char* upd = dres(P.update.p, argtab);
  char* out = dres(P.out, argtab);
  if (P.in_place) {
    int64_t nu = 1;
    for (int d = 0; d < P.rank; ++d) nu *= P.upd_shape[d];
    if (P.has_undo) {
      // undo record: clamped start indices, then the window's previous values
      char* ub = dres(P.undo, argtab);
      if (blockIdx.x == 0 && threadIdx.x < CLJXLA_MAXR) ((int64_t*)ub)[threadIdx.x] = threadIdx.x < P.rank ? st[threadIdx.x] : 0;
      char* old = ub + 8 * CLJXLA_MAXR;
      for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nu; e += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = e, oo = 0, ostride = 1;
        for (int d = P.rank - 1; d >= 0; --d) {
          int64_t i = rem % P.upd_shape[d];
          rem /= P.upd_shape[d];
          oo += (st[d] + i) * ostride;
          ostride *= P.out_shape[d];
        }
        st_elem(old, e, P.dt, ld_elem(out, oo, P.dt));  // same thread reads old then writes new
        st_elem(out, oo, P.dt, ld_elem(upd, view_off(P.update, e), P.update.dt));
      }
      return;
    }
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nu; e += (int64_t)gridDim.x * blockDim.x) {
      int64_t rem = e, oo = 0, ostride = 1;
      for (int d = P.rank - 1; d >= 0; --d) {
        int64_t i = rem % P.upd_shape[d];
        rem /= P.upd_shape[d];
        oo += (st[d] + i) * ostride;
        ostride *= P.out_shape[d];
      }
      st_elem(out, oo, P.dt, ld_elem(upd, view_off(P.update, e), P.update.dt));
    }
    return;
  }
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < P.n; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = e, uo = 0;
    bool inside = true;
    int64_t ui = 0, ustride = 1;
    for (int d = P.rank - 1; d >= 0; --d) {
      int64_t i = rem % P.out_shape[d];
      rem /= P.out_shape[d];
      int64_t k = i - st[d];
      if (k < 0 || k >= P.upd_shape[d]) inside = false;
      ui += k * ustride;
      ustride *= P.upd_shape[d];
    }
    (void)uo;
    uint32_t v = inside ? ld_elem(upd, view_off(P.update, ui), P.update.dt)
                        : ld_elem(opnd, view_off(P.operand, e), P.operand.dt);
    st_elem(out, e, P.dt, v);
  }
}

struct UndoGeom {
  int rank, dt;
  int64_t out_shape[CLJXLA_MAXR], upd_shape[CLJXLA_MAXR];
};

__global__ void undo_apply_kernel(char* dst, const char* undo, UndoGeom G) {
  pdl_enter();
  const int64_t* st = (const int64_t*)undo;
  const char* old = undo + 8 * CLJXLA_MAXR;
  int64_t nu = 1;
  for (int d = 0; d < G.rank; ++d) nu *= G.upd_shape[d];
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nu; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = e, oo = 0, ostride = 1;
    for (int d = G.rank - 1; d >= 0; --d) {
      int64_t i = rem % G.upd_shape[d];
      rem /= G.upd_shape[d];
      int64_t s = st[d];
      s = s < 0 ? 0 : (s > G.out_shape[d] - G.upd_shape[d] ? G.out_shape[d] - G.upd_shape[d] : s);
      oo += (s + i) * ostride;
      ostride *= G.out_shape[d];
    }
    st_elem(dst, oo, G.dt, ld_elem(old, e, G.dt));
  }
}

inline int grid_for(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  if (g > 148 * 64) g = 148 * 64;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

void launch_ew(const EwParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.n == 0) return;
  launch_k(ew_kernel, dim3(grid_for(p.n, 256)), dim3(256), 0, s, 1, p, argtab);
}
static bool view_is_dense(const TView& v) {
  int64_t acc = 1;
  for (int d = v.rank - 1; d >= 0; --d) {
    if (v.shape[d] != 1 && v.stride[d] != acc) return false;
    acc *= v.shape[d];
  }
  return true;
}

void launch_copy(const CopyParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.n == 0) return;
  if (p.src.dt == p.dst.dt && view_is_dense(p.src) && view_is_dense(p.dst)) {
    const int64_t es = p.src.dt == KDT_F32 || p.src.dt == KDT_I32 || p.src.dt == KDT_U32 ? 4
                       : (p.src.dt == KDT_BF16 || p.src.dt == KDT_F16 || p.src.dt == KDT_I16) ? 2
                       : (p.src.dt == KDT_I64 || p.src.dt == KDT_F64) ? 8 : 1;
    const int64_t bytes = p.n * es;
    int vec = 1;
    if (bytes % 16 == 0 && p.src.p.off % 16 == 0 && p.dst.p.off % 16 == 0) vec = 16;
    else if (bytes % 4 == 0 && p.src.p.off % 4 == 0 && p.dst.p.off % 4 == 0) vec = 4;
    launch_k(copy_bytes_kernel, dim3(grid_for(bytes / vec, 256)), dim3(256), 0, s, 1, p.src.p, p.dst.p, bytes, vec, argtab);
    return;
  }
  launch_k(copy_kernel, dim3(grid_for(p.n, 256)), dim3(256), 0, s, 1, p, argtab);
}
void launch_reduce(const ReduceParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.n_out == 0) return;
  int64_t g = p.n_out < 148 * 32 ? p.n_out : 148 * 32;
  if (p.n_red >= 2048) launch_k(reduce_kernel<512>, dim3((int)g), dim3(512), 0, s, 1, p, argtab);
  else if (p.n_red >= 256) launch_k(reduce_kernel<256>, dim3((int)g), dim3(256), 0, s, 1, p, argtab);
  else launch_k(reduce_kernel<64>, dim3((int)g), dim3(64), 0, s, 1, p, argtab);
}
void launch_gather(const GatherParams& p, const uint64_t* argtab, cudaStream_t s) {
  if (p.n_rows == 0) return;
  int64_t g = p.n_rows < 65535 ? p.n_rows : 65535;
  launch_k(gather_kernel, dim3((int)g), dim3(128), 0, s, 1, p, argtab);
}
void launch_undo_apply(void* dst, const void* undo, int rank, const int64_t* out_shape, const int64_t* upd_shape,
                       int dt, cudaStream_t s) {
  UndoGeom G{};
  G.rank = rank;
  G.dt = dt;
  int64_t nu = 1;
  for (int d = 0; d < rank; ++d) {
    G.out_shape[d] = out_shape[d];
    G.upd_shape[d] = upd_shape[d];
    nu *= upd_shape[d];
  }
  if (nu == 0) return;
  launch_k(undo_apply_kernel, dim3(grid_for(nu, 256)), dim3(256), 0, s, 1, (char*)dst, (const char*)undo, G);
}

void launch_dus(const DusParams& p, const uint64_t* argtab, cudaStream_t s) {
  int64_t n = p.n;
  if (p.in_place) {
    n = 1;
    for (int d = 0; d < p.rank; ++d) n *= p.upd_shape[d];
  }
  if (n == 0) return;
  launch_k(dus_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, 1, p, argtab);
}

}  // namespace cljxla

namespace cljxla {
namespace {

__global__ void stream_hold_kernel(int64_t ns) {
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (int i = 0; i < (1 << 22); ++i) {  // bounded: ends after ns or 2^22 sleeps
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if ((int64_t)(t - t0) >= ns) break;
    __nanosleep(1000);
  }
}

}  // namespace

void launch_stream_hold(int64_t ns, cudaStream_t s) { stream_hold_kernel<<<1, 1, 0, s>>>(ns); }

}  // namespace cljxla
