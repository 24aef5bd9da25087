// Run-time-loaded NCCL (nccl.cc): what tensor-parallel clients need.
#pragma once

#include <string>

#include "common.h"
#include "kernels.h"

namespace cljxla {

std::string nccl_unique_id_hex();                                  // 256 hex characters
void* nccl_comm_init(int nranks, int rank, const std::string& id_hex);  // a collective over all ranks
void nccl_all_reduce_sum(const void* src, void* dst, size_t count, int kdt, void* comm, cudaStream_t s);
void nccl_comm_destroy(void* comm);

}  // namespace cljxla
