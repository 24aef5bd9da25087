// One-shot all-reduce over NVLink peer memory for the small per-layer
// activations of tensor-parallel decode (a [B, 1, d] vector per all_reduce op,
// gemma.clj attention and MLP blocks sharded by heads / columns).
//
// Every rank owns one exchange buffer, mapped into every other rank's address
// space through CUDA IPC:  data[2 phases][ranks][slot_bytes] | flags[2][ranks].
// A call (epoch e, phase e & 1) has one CTA per rank:
//   1. store the rank's operand into slot [phase][rank] of every rank's buffer
//      (its own included), fence at system scope;
//   2. publish e in flag [phase][rank] of every rank's buffer (release);
//   3. wait until every flag [phase][src] of its own buffer reads e (acquire;
//      bounded: on a timeout the error word is set and the sum is skipped);
//   4. sum the slots in rank order in f32 and round once to the element type,
//      so every rank holds the same bits (the reduction order the oracle uses).
// Two phases make reuse safe: a rank reaches call e + 2, which overwrites the
// phase-e slots, only after every rank has published call e + 1, which each
// does after finishing its own sum of call e.  The epoch counter lives on the
// device and advances inside the kernel, so graph replays need no host input.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include <algorithm>
#include <cstdlib>

#include "common.h"
#include "kernels.h"
#include "nccl_rt.h"

namespace cljxla {
namespace {

// polls before a wait gives up (P2PAllReduce::wait_polls): the first
// P2P_FAST_POLLS about 64 ns apart, then about 1 us apart, ~16 s in all by
// default (ranks reach their first call after compiling their own
// executables, which need not take the same time)
constexpr uint32_t P2P_FAST_POLLS = 1u << 14;
constexpr int P2P_THREADS = 1024;

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(P2P_THREADS) p2p_allreduce_kernel(const char* __restrict__ src, char* __restrict__ dst,
                                                                    int64_t count, int dt,
                                                                    const uint64_t* __restrict__ peers, int rank,
                                                                    int ranks, int64_t slot_bytes, unsigned* epoch,
                                                                    unsigned* err, uint32_t wait_polls) {
  __shared__ unsigned s_ep;
  __shared__ int s_ok;
  // launched as a programmatic dependent: resident before the producer of src
  // ends, and the launch after it may become resident early in turn
  pdl_enter();
  if (threadIdx.x == 0) {
    s_ep = *epoch + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned ep = s_ep;
  const int phase = (int)(ep & 1u);
  const int es = dt == KDT_F32 ? 4 : 2;
  const int64_t bytes = count * es;
  const int64_t flag_off = 2 * (int64_t)ranks * slot_bytes;
  // 1. the operand into slot [phase][rank] of every buffer (16-byte pieces; bytes % 16 == 0)
  const int64_t my_slot = ((int64_t)phase * ranks + rank) * slot_bytes;
  for (int p = 0; p < ranks; ++p) {
    char* to = (char*)(uintptr_t)peers[p] + my_slot;
    for (int64_t i = threadIdx.x; i * 16 < bytes; i += P2P_THREADS)
      *(uint4*)(to + i * 16) = *(const uint4*)(src + i * 16);
  }
  __threadfence_system();
  __syncthreads();
  // 2. publish
  if (threadIdx.x < ranks) {
    unsigned* f = (unsigned*)((char*)(uintptr_t)peers[threadIdx.x] + flag_off) + phase * ranks + rank;
    st_release_sys(f, ep);
  }
  // 3. wait for every source (bounded)
  if (threadIdx.x < ranks) {
    const unsigned* f = (const unsigned*)((const char*)(uintptr_t)peers[rank] + flag_off) + phase * ranks + threadIdx.x;
    uint32_t n = 0;
    while (ld_acquire_sys(f) != ep) {
      if (++n > wait_polls) {
        atomicOr(err, 1u);
        s_ok = 0;
        break;
      }
      __nanosleep(n < P2P_FAST_POLLS ? 64 : 1024);
    }
  }
  __syncthreads();
  // 4. rank-order sum from this rank's own buffer (not cached: the slots are rewritten every other call)
  if (s_ok) {
    const char* base = (const char*)(uintptr_t)peers[rank] + (int64_t)phase * ranks * slot_bytes;
    for (int64_t i = threadIdx.x; i < count; i += P2P_THREADS) {
      float acc = 0.f;
      for (int s = 0; s < ranks; ++s) {
        const char* sl = base + (int64_t)s * slot_bytes;
        acc += dt == KDT_F32 ? __ldcv((const float*)sl + i)
                             : __uint_as_float((uint32_t)__ldcv((const unsigned short*)sl + i) << 16);
      }
      if (dt == KDT_F32) ((float*)dst)[i] = acc;
      else ((__nv_bfloat16*)dst)[i] = __float2bfloat16_rn(acc);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *epoch = ep;
}

}  // namespace

P2PAllReduce::~P2PAllReduce() {
  for (void* p : opened)
    if (p) cudaIpcCloseMemHandle(p);
  if (d_peers) cudaFree(d_peers);
  if (d_epoch) cudaFree(d_epoch);
  if (local) cudaFree(local);
  if (h_err) cudaFreeHost(h_err);
}

std::string P2PAllReduce::export_handle(int ranks_, int rank_, int64_t slot) {
  if (ranks_ < 2 || ranks_ > P2P_MAX_RANKS || rank_ < 0 || rank_ >= ranks_ || slot < 16 || slot % 16)
    fail(E_INVALID, "bad one-shot all-reduce group");
  if (const char* e = getenv("CLJXLA_B200_P2P_WAIT_POLLS"))
    if (atoll(e) > 0) wait_polls = (uint32_t)std::min<long long>(atoll(e), 1LL << 30);
  if (!local) {
    ranks = ranks_;
    rank = rank_;
    slot_bytes = slot;
    const size_t total = (size_t)(2 * ranks * slot_bytes) + 2 * ranks * sizeof(unsigned);
    CUDA_OK(cudaMalloc(&local, total));
    CUDA_OK(cudaMemset(local, 0, total));
    CUDA_OK(cudaDeviceSynchronize());
  }
  cudaIpcMemHandle_t h;
  CUDA_OK(cudaIpcGetMemHandle(&h, local));
  static const char* hex = "0123456789abcdef";
  std::string s;
  const unsigned char* b = (const unsigned char*)&h;
  for (size_t i = 0; i < sizeof(h); ++i) s += hex[b[i] >> 4], s += hex[b[i] & 15];
  return s;
}

void P2PAllReduce::import_handles(const std::string& all) {
  const size_t hl = 2 * sizeof(cudaIpcMemHandle_t);
  if (!local || all.size() != hl * (size_t)ranks) fail(E_INVALID, "one-shot all-reduce handles do not match the group");
  uint64_t ptrs[P2P_MAX_RANKS] = {};
  for (int r = 0; r < ranks; ++r) {
    if (r == rank) {
      ptrs[r] = (uint64_t)(uintptr_t)local;
      continue;
    }
    cudaIpcMemHandle_t h;
    unsigned char* b = (unsigned char*)&h;
    for (size_t i = 0; i < sizeof(h); ++i) {
      auto nib = [&](char c) { return (unsigned char)(c <= '9' ? c - '0' : c - 'a' + 10); };
      b[i] = (unsigned char)(nib(all[r * hl + 2 * i]) << 4 | nib(all[r * hl + 2 * i + 1]));
    }
    void* p = nullptr;
    CUDA_OK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    opened.push_back(p);
    ptrs[r] = (uint64_t)(uintptr_t)p;
  }
  CUDA_OK(cudaMalloc((void**)&d_peers, sizeof(ptrs)));
  CUDA_OK(cudaMemcpy(d_peers, ptrs, sizeof(ptrs), cudaMemcpyHostToDevice));
  CUDA_OK(cudaMalloc((void**)&d_epoch, sizeof(unsigned)));
  CUDA_OK(cudaMemset(d_epoch, 0, sizeof(unsigned)));
  CUDA_OK(cudaHostAlloc((void**)&h_err, sizeof(unsigned), cudaHostAllocMapped));
  *h_err = 0;
  CUDA_OK(cudaHostGetDevicePointer((void**)&d_err, h_err, 0));
  CUDA_OK(cudaDeviceSynchronize());
  ready = true;
}

bool P2PAllReduce::fits(int64_t count, int dt) const {
  const int64_t bytes = count * (dt == KDT_F32 ? 4 : 2);
  return ready && (dt == KDT_F32 || dt == KDT_BF16) && bytes % 16 == 0 && bytes <= slot_bytes;
}

void P2PAllReduce::run(const void* src, void* dst, int64_t count, int dt, cudaStream_t s) {
  if (((uintptr_t)src | (uintptr_t)dst) & 15) fail(E_INTERNAL, "one-shot all-reduce operands not 16-byte aligned");
  launch_k(p2p_allreduce_kernel, dim3(1), dim3(P2P_THREADS), 0, s, 1, (const char*)src, (char*)dst, count, dt,
           (const uint64_t*)d_peers, rank, ranks, slot_bytes, d_epoch, d_err, wait_polls);
}

void P2PAllReduce::check() const {
  if (h_err && *(volatile unsigned*)h_err)
    fail(E_INTERNAL, "one-shot all-reduce: a peer did not arrive within the wait limit (group out of step)");
}

}  // namespace cljxla
