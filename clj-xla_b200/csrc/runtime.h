// Runtime objects behind the opaque PJRT handles.
//
// Buffers are versions of device storage.  Normally a buffer owns its storage
// (one version, the head).  A KV-cache dynamic_update_slice executed in place
// (planner.h InplaceDus) writes the new window into the argument's storage and
// returns a result buffer that becomes the storage's new head; the argument
// buffer keeps its PJRT meaning (inputs are not donated, pjrt.clj:478-480)
// through an undo record - the window's previous values - chained to the
// newer version.  Reading or re-using a stale buffer rebuilds its content into
// fresh storage (copy of the head, undo records applied newest first); a
// stale buffer the host destroys (the decode loop's old caches) costs nothing.
#pragma once

#include <atomic>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "ir.h"
#include "nccl_rt.h"
#include "planner.h"

struct PJRT_Error {
  int code;
  std::string msg;
};

struct PJRT_Device {
  int ordinal = 0;
};

struct PJRT_Client;

namespace cljxla {

struct Storage {
  PJRT_Client* client = nullptr;
  void* ptr = nullptr;
  size_t bytes = 0;
  ~Storage();
};

struct Version {
  std::shared_ptr<Storage> storage;
  std::shared_ptr<Version> newer;  // null: this version is the storage's current content
  void* undo = nullptr;            // undo record turning newer's content into this one's
  size_t undo_bytes = 0;
  int rank = 0;
  DT dt = DT::BF16;
  int64_t out_shape[CLJXLA_MAXR] = {}, upd_shape[CLJXLA_MAXR] = {};
  PJRT_Client* client = nullptr;
  ~Version();
};

}  // namespace cljxla

struct PJRT_Buffer {
  PJRT_Client* client = nullptr;
  cljxla::DT dt = cljxla::DT::F32;
  std::vector<int64_t> dims;
  size_t bytes = 0;
  std::shared_ptr<cljxla::Version> ver;
  void* ptr() const { return ver && ver->storage ? ver->storage->ptr : nullptr; }
  bool current() const { return !ver || !ver->newer; }
};

struct PJRT_Event {
  cudaEvent_t ev = nullptr;
  int code = 0;
  std::string msg;
};

namespace cljxla {

// One compiled plan with its argument table and captured graph.
struct ExecVariant {
  std::unique_ptr<Plan> plan;
  void* consts = nullptr;
  uint64_t* d_argtab = nullptr;
  std::vector<uint64_t> h_argtab;
  // tensor-map table (Plan::tmaps + status word): device copy, host image, and
  // the operand addresses the image was last encoded for
  void* d_tmaps = nullptr;
  std::vector<uint64_t> h_tmaps;
  std::vector<uint64_t> tmap_addr;
  unsigned* status_host = nullptr;  // pinned copy of the status word, refreshed after each run
  cudaGraphExec_t graph = nullptr;
  cudaGraph_t graph_def = nullptr;
  int runs = 0;
  bool graph_failed = false;
};

}  // namespace cljxla

struct PJRT_LoadedExecutable {
  PJRT_Client* client = nullptr;
  cljxla::ExecVariant copy;     // results in fresh buffers
  cljxla::ExecVariant inplace;  // KV updates in place (when the graph has any); plan null otherwise
  void* arena = nullptr;        // scratch shared by both variants (never active together)
  size_t arena_bytes = 0;
  const cljxla::Plan& plan() const { return *copy.plan; }
};

struct ClientOptions {
  int device = -1;
  bool fuse = true;
  bool fast_kernels = true;
  bool cuda_graphs = true;
  bool kv_in_place = true;
  // tensor parallelism: this client is rank tp_rank of tp_size, joined through
  // the NCCL unique id tp_nccl_id (hex) that every rank was given
  int tp_size = 1, tp_rank = 0;
  std::string tp_nccl_id;
  // cap on the device memory this client holds (buffers, undo records, executable
  // scratch); 0 = no cap.  A request past it fails with RESOURCE_EXHAUSTED.
  int64_t memory_limit = 0;
};

struct PJRT_Client {
  ClientOptions opt;
  PJRT_Device device;
  PJRT_Device* device_list[1] = {&device};
  cudaStream_t stream = nullptr;
  std::mutex mu;
  // pinned staging for large device-to-host reads (grown on demand)
  void* pinned = nullptr;
  size_t pinned_bytes = 0;
  // pinned staging ring for large host-to-device uploads (weights): the host
  // copies chunk i + 1 into one buffer while the DMA engine reads chunk i
  void* up_stage[2] = {nullptr, nullptr};
  cudaEvent_t up_done[2] = {nullptr, nullptr};
  std::string platform = "cuda";
  void* nccl_comm = nullptr;  // tp_size > 1
  std::atomic<int64_t> held_bytes{0};  // device memory held through client_alloc
  // freed blocks of at most kSmallBlock bytes, by rounded size, reused by the
  // next allocation of that size (every use is ordered on the client's stream):
  // a decode step's undo records and result buffers cost no allocator call.
  // They stay in held_bytes while cached.
  static constexpr size_t kSmallBlock = 4u << 20;
  std::mutex small_mu;
  std::map<size_t, std::vector<void*>> small_free;
  cljxla::P2PAllReduce* p2p = nullptr;  // one-shot peer all-reduce, once its handles are exchanged
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

// Stream-ordered device allocation charged to the client (its memory_limit
// applies; RESOURCE_EXHAUSTED past it or when the device is out of memory),
// and its release.
void* client_alloc(PJRT_Client* c, size_t bytes);
void client_free(PJRT_Client* c, void* p, size_t bytes);
// returns the cached small blocks to the device allocator (client teardown)
void client_release_cached(PJRT_Client* c);

// New head-version buffer over fresh storage of `bytes` (stream-ordered allocation).
PJRT_Buffer* new_buffer(PJRT_Client* c, DT dt, const std::vector<int64_t>& dims);
// Rebuilds a stale buffer's content into fresh storage so it becomes a head.
void ensure_current(PJRT_Buffer* b);
void exec_run(PJRT_LoadedExecutable* ex, PJRT_Buffer* const* args, size_t nargs, PJRT_Buffer** outs);
void setup_variant(ExecVariant& v, void* arena);
void destroy_variant(ExecVariant& v);

}  // namespace cljxla
