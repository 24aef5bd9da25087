// Runtime objects behind the opaque PJRT handles.
#pragma once

#include <atomic>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "ir.h"
#include "planner.h"

struct PJRT_Error {
  int code;
  std::string msg;
};

struct PJRT_Device {
  int ordinal = 0;
};

struct PJRT_Client;

struct PJRT_Buffer {
  PJRT_Client* client = nullptr;
  cljxla::DT dt = cljxla::DT::F32;
  std::vector<int64_t> dims;
  void* ptr = nullptr;   // device memory (owned unless `alias` is set)
  size_t bytes = 0;
  bool owned = true;
  size_t nbytes() const { return bytes; }
};

struct PJRT_Event {
  cudaEvent_t ev = nullptr;
  int code = 0;
  std::string msg;
};

struct PJRT_LoadedExecutable {
  PJRT_Client* client = nullptr;
  std::unique_ptr<cljxla::Plan> plan;
  void* arena = nullptr;
  void* consts = nullptr;
  uint64_t* d_argtab = nullptr;
  std::vector<uint64_t> h_argtab;
  cudaGraphExec_t graph = nullptr;
  cudaGraph_t graph_def = nullptr;
  int runs = 0;
  bool graph_failed = false;
  std::string hash;
};

struct ClientOptions {
  int device = -1;
  bool fuse = true;
  bool fast_kernels = true;
  bool cuda_graphs = true;
  bool kv_in_place = false;
};

struct PJRT_Client {
  ClientOptions opt;
  PJRT_Device device;
  PJRT_Device* device_list[1] = {&device};
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::string platform = "cuda";
};

namespace cljxla {

struct ProfileEntry {
  std::string kind, label;
  double ms = 0;
  int64_t calls = 0;
  int64_t bytes = 0, flops = 0;
};

struct ProfileState {
  bool enabled = false;
  std::map<std::string, ProfileEntry> entries;
};
ProfileState& profile_state();

void exec_run(PJRT_LoadedExecutable* ex, PJRT_Buffer* const* args, size_t nargs, PJRT_Buffer** outs);

}  // namespace cljxla
