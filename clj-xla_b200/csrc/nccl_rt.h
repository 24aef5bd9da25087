// Run-time-loaded NCCL (nccl.cc): what tensor-parallel clients need.
#pragma once

#include <string>
#include <vector>

#include "common.h"
#include "kernels.h"

namespace cljxla {

std::string nccl_unique_id_hex();                                  // 256 hex characters
void* nccl_comm_init(int nranks, int rank, const std::string& id_hex);  // a collective over all ranks
// reduce: RED_ADD (sum) or RED_MAX (elementwise maximum; also for i32)
void nccl_all_reduce(const void* src, void* dst, size_t count, int kdt, int reduce, void* comm, cudaStream_t s);
void nccl_comm_destroy(void* comm);

// One-shot all-reduce over NVLink peer memory (p2p_allreduce.cu) for messages
// up to slot_bytes: each rank's exchange buffer is shared through CUDA IPC.
constexpr int P2P_MAX_RANKS = 8;
struct P2PAllReduce {
  int ranks = 0, rank = 0;
  int64_t slot_bytes = 0;
  void* local = nullptr;             // this rank's exchange buffer
  std::vector<void*> opened;         // peers' buffers mapped here
  uint64_t* d_peers = nullptr;       // device array of every rank's buffer address
  unsigned* d_epoch = nullptr;       // calls completed (advanced by the kernel)
  unsigned* h_err = nullptr;         // mapped host word: a wait ran out
  unsigned* d_err = nullptr;
  // polls before a wait gives up (CLJXLA_B200_P2P_WAIT_POLLS; default 2^24, ~16 s)
  uint32_t wait_polls = 1u << 24;
  bool ready = false;
  ~P2PAllReduce();
  std::string export_handle(int ranks, int rank, int64_t slot_bytes);  // allocates on first use
  void import_handles(const std::string& all_ranks_hex);               // every rank's handle, rank order
  bool fits(int64_t count, int dt) const;
  void run(const void* src, void* dst, int64_t count, int dt, cudaStream_t s);
  void check() const;  // fails if a previous call's wait ran out
};

}  // namespace cljxla
