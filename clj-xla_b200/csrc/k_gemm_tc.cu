// Prefill and batched-decode dot_general on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA).
//
// C[M, N] = A[M, K] . B[N, K]^T with bf16 operands, f32 accumulation in tensor
// memory and the result rounded once to the printed type (bf16 or f32).  This
// is the shape of every Gemma linear layer and LM head in a prefill graph: the
// activations [B*S, K] times a weight printed as transpose([N, K])
// (gemma.clj:8-23, :131-133, :272-273), both operands K-contiguous.
//
// Persistent kernel, one CTA per SM, 192 threads in three roles:
//   warp 0 (one lane)   TMA producer: 128x64 A tile + 256x64 B tile per stage
//                       into a 4-stage shared-memory ring (128-byte swizzle);
//   warp 1 (one lane)   MMA issuer: 4 x tcgen05.mma (M=128, N=256, K=16) per
//                       stage into one of two 128x256 f32 TMEM accumulators;
//                       tcgen05.commit frees the stage / publishes the tile;
//   warps 2-5           epilogue: tcgen05.ld of the accumulator (each warp its
//                       32-lane quarter), round, store; the other accumulator
//                       is meanwhile being filled for the next tile.
// Tiles are walked M-fastest so CTAs running at the same time share the weight
// tile (read from HBM once) while the small activation matrix stays in L2.
//
// Batched decode (at most 64 rows of A; a few hundred bytes of activations
// against megabytes of weights): the weight matrix is the stream, so the tile
// is 64 weight rows wide (MMA N = 64) and a stage carries four 64-wide K
// blocks (512 contiguous bytes of every weight row, 3-5 stages in flight); A
// is copied for its own rows only (the MMA's other rows read stale shared
// memory and their results are never stored).  When the 64-row tiles leave
// SMs idle, each tile's K blocks are split over CTAs: a (tile, split) unit
// stores its f32 partial tile, and the last split of the tile to arrive (an
// acq_rel counter) sums the partials in split order and stores C, so the
// result does not depend on which CTA finishes first.
//
// f32 activations times a bf16 weight (the attention-output projection of a
// Gemma prefill, whose context vectors are f32): the activation is first split
// exactly into three bf16 planes x = hi + mid + lo (8 + 8 + 8 significand
// bits), and the k-loop runs over the three planes against the same weight
// tiles, accumulating hi.w + mid.w + lo.w in one f32 accumulator.
//
// Tensor maps live in a per-executable device table that the executor
// re-encodes when the operand addresses change; the producer acquires them
// through the tensormap proxy before the first copy.  Every mbarrier wait is
// bounded: on a timeout the kernel records it in the status word, lets its own
// copies and MMAs drain, frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "fast_kernels.h"

namespace cljxla {
namespace {

constexpr int BM = 128, BK = 64;
constexpr int THREADS = 192;
constexpr int MAX_STAGES = 8;
constexpr int STAGE_BUDGET = 196 * 1024;  // shared memory for the stage ring
constexpr uint32_t WAIT_LIMIT = 1u << 22;  // try_wait rounds before a wait is declared failed

// Tile shapes: N = 256 for prefill (one 64-wide K block per stage, 4
// stages); N = 64 for at most 64 rows of A (batched decode, where the weight
// tile is the stream): four K blocks per stage, so each weight row is read
// 512 contiguous bytes at a time, with the K blocks split over CTAs.
template <int BN_>
struct TcShape {
  static constexpr int KSUB = BN_ == 256 ? 1 : 4;  // 64-wide K blocks per stage
  static constexpr int B_SUB = BN_ * BK * 2;      // one K block of the B tile
  static constexpr int B_STAGE = KSUB * B_SUB;
  static constexpr uint32_t TMEM_COLS = 2 * BN_;  // two f32 accumulators of 128 lanes x BN_ columns
  // kind::f16 instruction descriptor: D f32, A/B bf16, both K-major, N = BN_, M = 128
  static constexpr uint32_t IDESC =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN_ >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  // A rows per copy a_box (a multiple of 8): bytes of a stage's A sub-tiles,
  // ring depth and dynamic shared memory (host and device agree)
  __host__ __device__ static constexpr int a_stage(int a_box) { return KSUB * a_box * BK * 2; }
  __host__ __device__ static constexpr int stages(int a_box) {
    return BN_ == 256 ? 4 : (STAGE_BUDGET / (a_stage(a_box) + B_STAGE) < MAX_STAGES ? STAGE_BUDGET / (a_stage(a_box) + B_STAGE) : MAX_STAGES);
  }
  __host__ __device__ static constexpr int smem_bytes(int a_box) {
    return stages(a_box) * (a_stage(a_box) + B_STAGE) + 1024 /* alignment slack */ + 256 /* barriers */;
  }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_expect_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// waits until the phase with the given parity has completed; false after WAIT_LIMIT rounds
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
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

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// shared-memory matrix descriptor: K-major tile of 128-byte rows, 128-byte
// swizzle, 8-row groups 1024 bytes apart (tile base 1024-byte aligned)
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // descriptor version
  d |= (uint64_t)2 << 61;             // 128-byte swizzle
  return d;
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// barrier over the four epilogue warps only (named barrier 1)
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// AND of p over the four epilogue warps (the same barrier): they leave their
// loop together, so no epilogue warp waits at epi_sync for one that left
__device__ __forceinline__ bool epi_all(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred q, o;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred o, 1, 128, q;\n\tselp.u32 %0, 1, 0, o;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

// rounds and stores 32 consecutive f32 values of row `row` of C from column col0
__device__ __forceinline__ void store_row32(char* C, const TcGemmParams& P, int64_t row, int64_t col0, const uint32_t* v) {
  if (P.c_dt == KDT_F32) {
    float* dst = (float*)C + row * P.N + col0;
    if (col0 + 32 <= P.N && (P.N % 4) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *(float4*)(dst + i) = make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]),
                                          __uint_as_float(v[i + 3]));
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < P.N) dst[i] = __uint_as_float(v[i]);
    }
  } else {
    __nv_bfloat16* dst = (__nv_bfloat16*)C + row * P.N + col0;
    if (col0 + 32 <= P.N && (P.N % 8) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 w;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(__uint_as_float(v[i]), __uint_as_float(v[i + 1]));
        __nv_bfloat162 h1 = __floats2bfloat162_rn(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
        __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(v[i + 4]), __uint_as_float(v[i + 5]));
        __nv_bfloat162 h3 = __floats2bfloat162_rn(__uint_as_float(v[i + 6]), __uint_as_float(v[i + 7]));
        w.x = *(uint32_t*)&h0;
        w.y = *(uint32_t*)&h1;
        w.z = *(uint32_t*)&h2;
        w.w = *(uint32_t*)&h3;
        *(uint4*)(dst + i) = w;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < P.N) dst[i] = __float2bfloat16_rn(__uint_as_float(v[i]));
    }
  }
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BN_>
__global__ void __launch_bounds__(THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcGemmParams P,
                                                             const uint64_t* __restrict__ argtab) {
  using SH = TcShape<BN_>;
  constexpr int KSUB = SH::KSUB;
  const int STAGES = SH::stages(P.a_box);
  const int A_STAGE = SH::a_stage(P.a_box), A_SUB = P.a_box * BK * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  // [stages][KSUB][A sub-tile of a_box rows] then [stages][KSUB][B sub-tile];
  // the MMA reads 128 rows of A from a sub-tile, the rows past a_box landing in
  // the next sub-tiles (or the B ring): their results are never stored
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE;
  uint64_t* full = (uint64_t*)(sB + STAGES * SH::B_STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2] accumulator ready
  uint64_t* tempty = tfull + 2;      // [2] accumulator drained by the epilogue
  uint64_t* drain = tempty + 2;      // MMA completion at exit
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  __shared__ int s_failed, s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (P.M + BM - 1) / BM, tiles_n = (P.N + BN_ - 1) / BN_;
  const int ntiles = tiles_m * tiles_n;
  const int kblocks = (P.K + BK - 1) / BK;
  const int kb_total = kblocks * (P.a_parts > 1 ? P.a_parts : 1);
  const int ks = P.ksplit > 1 ? P.ksplit : 1;
  const int nunits = ntiles * ks;  // work unit: (tile, K split); the host keeps ks <= kb_total
  const uint32_t tx_sub = (uint32_t)(A_SUB + SH::B_SUB);
  const char* tmA = dres(P.tmap_a, argtab);
  const char* tmB = dres(P.tmap_b, argtab);
  unsigned* status = (unsigned*)dres(P.status, argtab);
  // Set-up and, for a weight operand, the first stages of B go out before the
  // dependency wait (the tensor-map table is written by a host copy ahead of
  // every launch; weights by no launch); A, the predecessor's result, is
  // copied only after it.  Tensor memory may be taken while the predecessor
  // still runs: it frees its own when its CTAs end.
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    s_failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(SH::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (!(warp == 0 && lane == 0)) pdl_enter();  // (the producer waits after its early weight copies)

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(tmA) : "memory");
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(tmB) : "memory");
    int pre = 0;  // stages of the first unit whose B copies went out before the wait
    if (P.b_const && (int)blockIdx.x < nunits) {
      const int tile = blockIdx.x / ks, kc = blockIdx.x - tile * ks;
      const int kb0 = (int)((int64_t)kb_total * kc / ks), kb1 = (int)((int64_t)kb_total * (kc + 1) / ks);
      const int n0 = (tile / tiles_m) * BN_;
      for (int kb = kb0; kb < kb1 && pre < STAGES; kb += KSUB, ++pre) {
        const int nsub = kb1 - kb < KSUB ? kb1 - kb : KSUB;
        mbar_expect_only(&full[pre], (uint32_t)(nsub * SH::B_SUB));
        for (int j = 0; j < nsub; ++j) {
          const int kk = (kb + j) % kblocks;
          tma_load_2d(sB + pre * SH::B_STAGE + j * SH::B_SUB, tmB, &full[pre], kk * BK, n0);
        }
      }
    }
    pdl_enter();
    int stage = 0, st = 0;
    uint32_t phase = 0;
    uint32_t issued_parity[MAX_STAGES];
    bool issued[MAX_STAGES];
    // (early copies count as issued: they land before the CTA may exit, even
    // when a failure stops the loop before their A copies go out)
    for (int s = 0; s < MAX_STAGES; ++s) issued[s] = s < pre, issued_parity[s] = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
      const int tile = u / ks, kc = u - tile * ks;
      const int kb0 = (int)((int64_t)kb_total * kc / ks), kb1 = (int)((int64_t)kb_total * (kc + 1) / ks);
      const int m0 = (tile % tiles_m) * BM, n0 = (tile / tiles_m) * BN_;
      for (int kb = kb0; kb < kb1; kb += KSUB, ++st) {
        const bool b_out = st < pre;  // this stage's B is already on its way (first ring round)
        if (!b_out && !mbar_wait(&empty[stage], phase ^ 1)) { ok = false; break; }
        if (*(volatile int*)&s_failed) { ok = false; break; }
        const int nsub = kb1 - kb < KSUB ? kb1 - kb : KSUB;
        mbar_expect_tx(&full[stage], (b_out ? (uint32_t)A_SUB : tx_sub) * (uint32_t)nsub);
        for (int j = 0; j < nsub; ++j) {
          const int part = (kb + j) / kblocks, kk = kb + j - part * kblocks;
          tma_load_2d(sA + stage * A_STAGE + j * A_SUB, tmA, &full[stage], kk * BK, part * P.a_plane_rows + m0);
          if (!b_out) tma_load_2d(sB + stage * SH::B_STAGE + j * SH::B_SUB, tmB, &full[stage], kk * BK, n0);
        }
        issued[stage] = true;
        issued_parity[stage] = phase;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) {
      atomicOr(status, 1u);
      s_failed = 1;
    }
    // the copies this thread issued land before the CTA may exit
    for (int s = 0; s < STAGES; ++s)
      if (issued[s] && !mbar_wait(&full[s], issued_parity[s])) atomicOr(status, 2u);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    int stage = 0, acc = 0;
    uint32_t phase = 0, acc_phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
      const int tile = u / ks, kc = u - tile * ks;
      const int kb0 = (int)((int64_t)kb_total * kc / ks), kb1 = (int)((int64_t)kb_total * (kc + 1) / ks);
      (void)tile;
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(acc * BN_);
      for (int kb = kb0; kb < kb1; kb += KSUB) {
        if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
        tc_fence_after();
        const int nsub = kb1 - kb < KSUB ? kb1 - kb : KSUB;
        for (int i = 0; i < nsub; ++i) {
          const uint64_t ad = sw128_desc(smem_u32(sA + stage * A_STAGE + i * A_SUB));
          const uint64_t bd = sw128_desc(smem_u32(sB + stage * SH::B_STAGE + i * SH::B_SUB));
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)  // K=16 per MMA: 32 bytes further along the swizzled rows
            umma(d, ad + (uint64_t)(2 * j), bd + (uint64_t)(2 * j), SH::IDESC, (kb + i > kb0 || j > 0) ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      umma_commit(&tfull[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (!ok) {
      atomicOr(status, 4u);
      s_failed = 1;
    }
    // every MMA this thread issued has completed before tensor memory is freed
    umma_commit(drain);
    if (!mbar_wait(drain, 0)) atomicOr(status, 8u);
  } else if (warp >= 2) {
    // ---------------- epilogue
    const int q = warp & 3;  // the TMEM lane quarter this warp may access
    const int r_in_tile = q * 32 + lane;
    const int et = threadIdx.x - 64;  // 0 .. 127 over the epilogue warps
    int acc = 0;
    uint32_t acc_phase = 0;
    char* C = dres(P.c, argtab);
    float* part = ks > 1 ? (float*)dres(P.part, argtab) : nullptr;
    unsigned* ctrs = ks > 1 ? (unsigned*)dres(P.counters, argtab) : nullptr;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
      const int tile = u / ks, kc = u - tile * ks;
      const int m0 = (tile % tiles_m) * BM, n0 = (tile / tiles_m) * BN_;
      bool ready = mbar_wait(&tfull[acc], acc_phase);
      ready = ks > 1 ? epi_all(ready) : __all_sync(0xffffffffu, ready);
      if (!ready) {
        if (lane == 0) atomicOr(status, 16u);
        break;
      }
      tc_fence_after();
      const int64_t row = (int64_t)m0 + r_in_tile;
      for (int c = 0; c < BN_; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN_ + c), v);
        if (row < P.M) {
          const int64_t col0 = (int64_t)n0 + c;
          if (ks == 1) {
            store_row32(C, P, row, col0, v);
          } else {  // this K split's f32 partial
            float* dst = part + ((int64_t)kc * P.M + row) * P.N + col0;
            if (col0 + 32 <= P.N && (P.N % 4) == 0) {
#pragma unroll
              for (int i = 0; i < 32; i += 4)
                *(float4*)(dst + i) = make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                                  __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
            } else {
              for (int i = 0; i < 32; ++i)
                if (col0 + i < P.N) dst[i] = __uint_as_float(v[i]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      if (ks > 1) {
        // the last split of the tile to arrive sums the partials in split order
        __threadfence();
        epi_sync();
        if (et == 0) {
          unsigned old;
          asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctrs + tile) : "memory");
          s_last = old == (unsigned)(ks - 1);
        }
        epi_sync();
        if (s_last) {
          const int rows = min(BM, P.M - m0);
          const int64_t plane = (int64_t)P.M * P.N;
          if ((P.N % 4) == 0) {
            // four columns per group, four groups per thread in flight at once
            constexpr int G4 = BN_ / 4;
            const int ngrp = rows * G4;
            for (int g0 = et; g0 < ngrp; g0 += 4 * 128) {
              float4 acc[4];
              int64_t off[4];
              bool on[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int g = g0 + i * 128;
                const int64_t r = m0 + g / G4, col = n0 + (int64_t)(g % G4) * 4;
                on[i] = g < ngrp && col < P.N;
                off[i] = r * P.N + col;
                acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll 2
              for (int k = 0; k < ks; ++k)
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  if (on[i]) {
                    const float4 v = __ldcg((const float4*)(part + k * plane + off[i]));
                    acc[i].x += v.x;
                    acc[i].y += v.y;
                    acc[i].z += v.z;
                    acc[i].w += v.w;
                  }
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                if (!on[i]) continue;
                if (P.c_dt == KDT_F32) {
                  *(float4*)((float*)C + off[i]) = acc[i];
                } else {
                  __nv_bfloat162 h0 = __floats2bfloat162_rn(acc[i].x, acc[i].y);
                  __nv_bfloat162 h1 = __floats2bfloat162_rn(acc[i].z, acc[i].w);
                  uint2 w;
                  w.x = *(uint32_t*)&h0;
                  w.y = *(uint32_t*)&h1;
                  *(uint2*)((__nv_bfloat16*)C + off[i]) = w;
                }
              }
            }
          } else {
            for (int e = et; e < rows * BN_; e += 128) {
              const int64_t r = m0 + e / BN_, col = n0 + e % BN_;
              if (col >= P.N) continue;
              float sum = 0.f;
              for (int k = 0; k < ks; ++k) sum += __ldcg(part + k * plane + r * P.N + col);
              if (P.c_dt == KDT_F32) ((float*)C)[r * P.N + col] = sum;
              else ((__nv_bfloat16*)C)[r * P.N + col] = __float2bfloat16_rn(sum);
            }
          }
          if (et == 0) ctrs[tile] = 0u;  // ready for the next launch
        }
        epi_sync();  // s_last is read by every epilogue thread before the next unit rewrites it
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(SH::TMEM_COLS) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  if (!fn) fail(E_INTERNAL, "cuTensorMapEncodeTiled is not available from the driver");
  return fn;
}

}  // namespace

void encode_tmap_bf16(void* out128, const void* base, int64_t inner, int64_t outer, int64_t row_bytes, int box_inner,
                      int box_outer) {
  if (((uintptr_t)base & 15) || (row_bytes & 15) || inner < 1 || outer < 1)
    fail(E_INTERNAL, "tensor map operand not 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()((CUtensorMap*)out128, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(E_INTERNAL, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

void tc_gemm_tile_shape(int* bm, int* bn, int* bk) {
  *bm = BM;
  *bn = 256;
  *bk = BK;
}

void tc_gemm_choose(int64_t M, int64_t N, int64_t K, int sms, int* bn, int* a_box, int* ksplit) {
  *bn = 256;
  *a_box = BM;
  *ksplit = 1;
  if (M > BM) return;  // prefill: whole 128 x 256 tiles
  // a few rows of A (batched decode): the weight matrix B is the stream, so
  // up to 64 rows take tiles 64 weight rows wide, and when the tiles leave SMs
  // idle the K blocks are split over CTAs (at least 4 blocks per split; units
  // = tiles x splits stay within one round over the SMs)
  if (M <= 64) {
    *bn = 64;
    *a_box = (int)((M + 7) / 8 * 8);
  }
  const int64_t tiles = (N + *bn - 1) / *bn, kblocks = (K + BK - 1) / BK;
  if (tiles < sms) *ksplit = (int)std::max<int64_t>(1, std::min<int64_t>(sms / tiles, kblocks / 4));
}

void launch_tc_gemm(const TcGemmParams& p, const uint64_t* argtab, cudaStream_t s) {
  const int sms = device_sm_count();
  const int bn = p.bn == 64 ? 64 : 256;
  const int64_t units = ((p.M + BM - 1) / BM) * ((p.N + bn - 1) / bn) * (int64_t)(p.ksplit > 1 ? p.ksplit : 1);
  const int grid = (int)(units < sms ? units : sms);
  if (grid <= 0) return;
  if (bn == 64) {
    const int smem = TcShape<64>::smem_bytes(p.a_box);
    ensure_smem_optin((const void*)tc_gemm_kernel<64>, smem);
    launch_k(tc_gemm_kernel<64>, dim3(grid), dim3(THREADS), smem, s, 1, p, argtab);
  } else {
    const int smem = TcShape<256>::smem_bytes(p.a_box);
    ensure_smem_optin((const void*)tc_gemm_kernel<256>, smem);
    launch_k(tc_gemm_kernel<256>, dim3(grid), dim3(THREADS), smem, s, 1, p, argtab);
  }
}

bool make_tc_gemm(const GemmParams& g, TcGemmParams& t) {
  if (g.batch != 1 || g.a_dt != KDT_BF16 || g.b_dt != KDT_BF16) return false;
  if (!(g.c_dt == KDT_BF16 || g.c_dt == KDT_F32)) return false;
  if (g.a_sk != 1 || g.b_sk != 1) return false;  // both operands K-contiguous
  if (g.M < 1 || g.N < 16 || g.K < 16) return false;
  if (g.M > (1 << 30) || g.N > (1 << 30) || g.K > (1 << 30)) return false;
  // TMA: 16-byte aligned bases and row strides
  if ((g.a.off % 16) || (g.b.off % 16) || (g.c.off % 16) || ((g.a_sm * 2) % 16) || ((g.b_sn * 2) % 16)) return false;
  if (g.a_sm < g.K || g.b_sn < g.K) return false;
  t = TcGemmParams{};
  t.c = g.c;
  t.a = g.a;
  t.b = g.b;
  t.M = (int32_t)g.M;
  t.N = (int32_t)g.N;
  t.K = (int32_t)g.K;
  t.c_dt = g.c_dt;
  t.a_ld = g.a_sm;
  t.b_ld = g.b_sn;
  t.a_parts = 1;
  t.a_plane_rows = t.M;
  t.bn = 256;
  t.a_box = BM;
  t.ksplit = 1;
  return true;
}

bool make_tc_gemm_split(const GemmParams& g, TcGemmParams& t) {
  // A: the dense [3 * M, K] bf16 planes of the split f32 activation (placed by the caller)
  if (g.batch != 1 || g.a_dt != KDT_F32 || g.b_dt != KDT_BF16) return false;
  if (!(g.c_dt == KDT_BF16 || g.c_dt == KDT_F32)) return false;
  if (g.b_sk != 1 || g.M < 16 || g.N < 16 || g.K < 16 || (g.K % 8)) return false;
  if (3 * g.M > (1 << 30) || g.N > (1 << 30) || g.K > (1 << 30)) return false;
  if ((g.b.off % 16) || (g.c.off % 16) || ((g.b_sn * 2) % 16) || g.b_sn < g.K) return false;
  t = TcGemmParams{};
  t.c = g.c;
  t.b = g.b;
  t.M = (int32_t)g.M;
  t.N = (int32_t)g.N;
  t.K = (int32_t)g.K;
  t.c_dt = g.c_dt;
  t.a_ld = g.K;
  t.b_ld = g.b_sn;
  t.a_parts = 3;
  t.a_plane_rows = t.M;
  t.bn = 256;
  t.a_box = BM;
  t.ksplit = 1;
  return true;
}

void verify_tc_gemm(const TcGemmParams& p, const RegionFn& region) {
  if (!(p.a_parts == 1 || p.a_parts == 3) || p.a_plane_rows != p.M) fail(E_INTERNAL, "bad tensor-core GEMM planes");
  region(p.a, ((int64_t)(p.a_parts * p.M - 1) * p.a_ld + p.K) * 2, "lhs");
  region(p.b, ((int64_t)(p.N - 1) * p.b_ld + p.K) * 2, "rhs");
  region(p.c, (int64_t)p.M * p.N * (int64_t)dt_size((DT)p.c_dt), "result");
  region(p.tmap_a, 128, "lhs tensor map");
  region(p.tmap_b, 128, "rhs tensor map");
  region(p.status, 4, "status word");
  const int64_t kb_total = (p.K + BK - 1) / BK * (int64_t)p.a_parts;
  if (!(p.bn == 256 || p.bn == 64) || p.a_box < 8 || p.a_box > BM || (p.a_box % 8) || p.ksplit < 1 ||
      p.ksplit > kb_total || (p.bn == 256 && p.a_box != BM) || (p.bn == 64 && p.a_box > 64) ||
      (p.bn == 64 ? TcShape<64>::smem_bytes(p.a_box) : TcShape<256>::smem_bytes(p.a_box)) > 227 * 1024)
    fail(E_INTERNAL, "bad tensor-core GEMM tiling");
  if (p.a_box < BM && p.a_box < p.M) fail(E_INTERNAL, "tensor-core GEMM rows beyond the A copy");
  if (p.ksplit > 1) {
    region(p.part, (int64_t)p.ksplit * p.M * p.N * 4, "split-K partials");
    region(p.counters, 4LL * ((p.M + BM - 1) / BM) * ((p.N + p.bn - 1) / p.bn), "split-K counters");
  }
}

}  // namespace cljxla
