// Executes a launch plan: refresh the dynamic part of the argument table,
// replay the captured CUDA graph (or launch eagerly the first time / when
// profiling).  Also owns buffer storage and the version chains of in-place
// KV updates (runtime.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "fast_kernels.h"
#include "jit.h"
#include "nccl_rt.h"
#include "runtime.h"

namespace cljxla {

Counters& counters() {
  static Counters c;
  return c;
}

namespace {
std::mutex g_dev_mu;
std::map<int, int> g_dev_sms;
std::map<std::pair<const void*, int>, int> g_smem_optin;

int current_device() {
  int dev = 0;
  CUDA_OK(cudaGetDevice(&dev));
  return dev;
}
}  // namespace

int device_sm_count() {
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  auto it = g_dev_sms.find(dev);
  if (it != g_dev_sms.end()) return it->second;
  int v = 0;
  CUDA_OK(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
  if (v <= 0) fail(E_INTERNAL, "device reports no multiprocessors");
  g_dev_sms[dev] = v;
  return v;
}

void ensure_smem_optin(const void* kernel, int bytes) {
  // also below 48 KB: the default limit is 48 KB less the kernel's static shared memory
  if (bytes <= 0) return;
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  int& have = g_smem_optin[{kernel, dev}];
  if (have >= bytes) return;
  CUDA_OK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  have = bytes;
}

ProfileState& profile_state() {
  static ProfileState p;
  return p;
}

void* client_alloc(PJRT_Client* c, size_t bytes) {
  if (!bytes) return nullptr;
  if (bytes <= PJRT_Client::kSmallBlock) {
    bytes = (bytes + 255) & ~(size_t)255;
    std::lock_guard<std::mutex> lk(c->small_mu);
    auto it = c->small_free.find(bytes);
    if (it != c->small_free.end() && !it->second.empty()) {
      void* p = it->second.back();
      it->second.pop_back();
      return p;
    }
  }
  const int64_t lim = c->opt.memory_limit;
  const int64_t now = c->held_bytes.fetch_add((int64_t)bytes) + (int64_t)bytes;
  if (lim > 0 && now > lim) {
    c->held_bytes.fetch_sub((int64_t)bytes);
    fail(E_OOM, "RESOURCE_EXHAUSTED: allocating " + std::to_string(bytes) + " bytes would hold " +
                    std::to_string(now) + " bytes, above the client's memory_limit_bytes " + std::to_string(lim));
  }
  void* p = nullptr;
  cudaError_t e = cudaMallocAsync(&p, bytes, c->stream);
  if (e != cudaSuccess) {
    c->held_bytes.fetch_sub((int64_t)bytes);
    cudaGetLastError();
    fail(e == cudaErrorMemoryAllocation ? E_OOM : E_INTERNAL,
         std::string(e == cudaErrorMemoryAllocation ? "RESOURCE_EXHAUSTED: " : "") + "device allocation of " +
             std::to_string(bytes) + " bytes failed: " + cudaGetErrorString(e));
  }
  return p;
}

void client_free(PJRT_Client* c, void* p, size_t bytes) {
  if (!p) return;
  if (bytes <= PJRT_Client::kSmallBlock) {  // kept for the next allocation of this size
    std::lock_guard<std::mutex> lk(c->small_mu);
    c->small_free[(bytes + 255) & ~(size_t)255].push_back(p);
    return;
  }
  cudaFreeAsync(p, c->stream);  // stream ordered after every reader
  c->held_bytes.fetch_sub((int64_t)bytes);
}

void client_release_cached(PJRT_Client* c) {
  std::lock_guard<std::mutex> lk(c->small_mu);
  for (auto& kv : c->small_free)
    for (void* p : kv.second) {
      cudaFreeAsync(p, c->stream);
      c->held_bytes.fetch_sub((int64_t)kv.first);
    }
  c->small_free.clear();
}

Storage::~Storage() { client_free(client, ptr, bytes); }

Version::~Version() { client_free(client, undo, undo_bytes); }

PJRT_Buffer* new_buffer(PJRT_Client* c, DT dt, const std::vector<int64_t>& dims) {
  auto* b = new PJRT_Buffer();
  b->client = c;
  b->dt = dt;
  b->dims = dims;
  b->bytes = (size_t)numel(dims) * dt_size(dt);
  auto st = std::make_shared<Storage>();
  st->client = c;
  st->bytes = b->bytes;
  if (b->bytes) {
    try {
      st->ptr = client_alloc(c, b->bytes);
    } catch (...) {
      st->ptr = nullptr;
      delete b;
      throw;
    }
  }
  b->ver = std::make_shared<Version>();
  b->ver->storage = st;
  b->ver->client = c;
  return b;
}

void ensure_current(PJRT_Buffer* b) {
  if (b->current()) return;
  // versions from b up to (not including) the head
  std::vector<Version*> chain;
  for (Version* v = b->ver.get(); v->newer; v = v->newer.get()) chain.push_back(v);
  PJRT_Client* c = b->client;
  auto st = std::make_shared<Storage>();
  st->client = c;
  st->bytes = b->bytes;
  if (b->bytes) {
    st->ptr = client_alloc(c, b->bytes);
    CUDA_OK(cudaMemcpyAsync(st->ptr, b->ver->storage->ptr, b->bytes, cudaMemcpyDeviceToDevice, c->stream));
    for (size_t i = chain.size(); i-- > 0;) {
      Version* v = chain[i];
      launch_undo_apply(st->ptr, v->undo, v->rank, v->out_shape, v->upd_shape, (int)v->dt, c->stream);
    }
    CUDA_OK(cudaGetLastError());
  }
  auto nv = std::make_shared<Version>();
  nv->storage = st;
  nv->client = c;
  b->ver = nv;  // the old version node stays in the chain for older buffers
}

void prepare_jit(Plan& p) {
  if (!jit_enabled()) return;
  std::vector<std::string> src;
  std::vector<Launch*> targets;
  for (Launch& l : p.launches) {
    std::string s;
    if (!jit_describe(l, &s, &l.jit_grid, &l.jit_block, &l.jit_cluster, &l.jit_args, &l.jit_smem)) continue;
    src.push_back(std::move(s));
    targets.push_back(&l);
  }
  std::vector<void*> fns = jit_compile(src);
  p.n_jit_missing = 0;
  for (size_t i = 0; i < targets.size(); ++i) {
    targets[i]->jit_fn = fns[i];
    if (!fns[i]) ++p.n_jit_missing;
  }
}

namespace {
// the collective context of the executable being launched on this thread
struct CollectiveCtx {
  void* comm = nullptr;
  P2PAllReduce* p2p = nullptr;
  int ranks = 1;
  const uint64_t* host_argtab = nullptr;
};
thread_local CollectiveCtx g_coll;
}  // namespace

void run_launch(const Launch& l, const uint64_t* argtab, cudaStream_t s) {
  const void* b = l.blob.data();
  if (l.kind == K_ALLREDUCE) {
    const AllReduceParams& a = *(const AllReduceParams*)b;
    if (!g_coll.comm) fail(E_PRECOND, "all_reduce in a graph run by a client without a tensor-parallel group");
    if (a.ranks != g_coll.ranks)
      fail(E_INVALID, "all_reduce over " + std::to_string(a.ranks) + " ranks on a client of " +
                          std::to_string(g_coll.ranks));
    const char* src = (const char*)(uintptr_t)(g_coll.host_argtab[a.src.slot] + (uint64_t)a.src.off);
    char* dst = (char*)(uintptr_t)(g_coll.host_argtab[a.dst.slot] + (uint64_t)a.dst.off);
    // the one-shot peer kernel sums; maxima (the vocab-split greedy token) go to NCCL
    if (a.reduce == RED_ADD && g_coll.p2p && g_coll.p2p->fits(a.count, a.dt)) g_coll.p2p->run(src, dst, a.count, a.dt, s);
    else nccl_all_reduce(src, dst, (size_t)a.count, a.dt, a.reduce, g_coll.comm, s);
    return;
  }
  if (l.jit_fn) {
    jit_launch(l.jit_fn, l.jit_grid, l.jit_block, l.jit_cluster, l.jit_smem, argtab, l.jit_args, s);
    return;
  }
  if ((!l.epi.empty() || !l.gtail.empty()) && (l.kind == K_GEMV || l.kind == K_GEMV_FUSED)) {
    // not compiled: the GEMV (its producer first), then the epilogue and group-tail programs
    if (l.kind == K_GEMV_FUSED) run_launch(l.parts[0], argtab, s);
    launch_gemv(*(const GemvParams*)b, argtab, s);
    for (const Launch& e : l.epi) run_launch(e, argtab, s);
    for (const Launch& q : l.gtail) run_launch(q, argtab, s);
    return;
  }
  if (!l.epi.empty()) {  // not compiled: the program, then its epilogue as its own launch
    Launch base = l;
    base.epi.clear();
    run_launch(base, argtab, s);
    for (const Launch& e : l.epi) run_launch(e, argtab, s);
    return;
  }
  if (l.kind == K_GEMV_FUSED) {  // not compiled: the producer in full, then the GEMV reading its x
    run_launch(l.parts[0], argtab, s);
    launch_gemv(*(const GemvParams*)b, argtab, s);
    return;
  }
  if (l.kind == K_GEMV_TAIL) {  // not compiled: the GEMV, then its tail programs one after another
    launch_gemv(*(const GemvParams*)b, argtab, s);
    for (const Launch& part : l.parts) run_launch(part, argtab, s);
    return;
  }
  if (l.kind == K_MULTI || l.kind == K_FUSED_DUS) {  // not compiled: the parts one after another
    for (const Launch& part : l.parts) run_launch(part, argtab, s);
    return;
  }
  switch (l.kind) {
    case K_EW: launch_ew(*(const EwParams*)b, argtab, s); break;
    case K_REDUCE: launch_reduce(*(const ReduceParams*)b, argtab, s); break;
    case K_COPY: launch_copy(*(const CopyParams*)b, argtab, s); break;
    case K_GATHER: launch_gather(*(const GatherParams*)b, argtab, s); break;
    case K_DUS: launch_dus(*(const DusParams*)b, argtab, s); break;
    case K_GEMM: launch_gemm(*(const GemmParams*)b, argtab, s); break;
    case K_ROWNORM: launch_row(*(const RowParams*)b, argtab, s); break;
    default: run_fast_launch(l, argtab, s); break;
  }
}

void setup_variant(ExecVariant& v, void* arena) {
  Plan& p = *v.plan;
  if (!p.const_blob.empty()) {
    CUDA_OK(cudaMalloc(&v.consts, p.const_blob.size()));
    CUDA_OK(cudaMemcpy(v.consts, p.const_blob.data(), p.const_blob.size(), cudaMemcpyHostToDevice));
  }
  v.h_argtab.assign((size_t)p.argtab_size(), 0);
  v.h_argtab[p.const_slot()] = (uint64_t)(uintptr_t)v.consts;
  for (size_t b = 0; b < p.tmp_offsets.size(); ++b)
    v.h_argtab[p.tmp_slot0() + b] = (uint64_t)(uintptr_t)arena + (uint64_t)p.tmp_offsets[b];
  if (p.has_table()) {
    CUDA_OK(cudaMalloc(&v.d_tmaps, (size_t)p.tmap_table_bytes()));
    CUDA_OK(cudaMemset(v.d_tmaps, 0, (size_t)p.tmap_table_bytes()));
    CUDA_OK(cudaMallocHost(&v.status_host, sizeof(unsigned)));
    *v.status_host = 0;
    v.h_tmaps.assign((size_t)p.tmap_table_bytes() / 8, 0);
    v.tmap_addr.assign(p.tmaps.size(), ~0ull);
    v.h_argtab[p.tmap_slot()] = (uint64_t)(uintptr_t)v.d_tmaps;
  }
  CUDA_OK(cudaMalloc(&v.d_argtab, v.h_argtab.size() * 8));
  CUDA_OK(cudaMemcpy(v.d_argtab, v.h_argtab.data(), v.h_argtab.size() * 8, cudaMemcpyHostToDevice));
}

void destroy_variant(ExecVariant& v) {
  if (v.graph) cudaGraphExecDestroy(v.graph);
  if (v.graph_def) cudaGraphDestroy(v.graph_def);
  if (v.consts) cudaFree(v.consts);
  if (v.d_argtab) cudaFree(v.d_argtab);
  if (v.d_tmaps) cudaFree(v.d_tmaps);
  if (v.status_host) cudaFreeHost(v.status_host);
  v = ExecVariant();
}

namespace {

// Re-encodes the tensor maps whose operand address changed since the last run
// and uploads the table (stream-ordered before the run's kernels).
void refresh_tmaps(ExecVariant& v, cudaStream_t s) {
  const Plan& p = *v.plan;
  if (!p.has_table()) return;
  if (*v.status_host)
    fail(E_INTERNAL, "a bounded wait in a kernel (tensor-core GEMM or bulk-copy GEMV) timed out in an earlier "
                     "execution (status " + std::to_string(*v.status_host) + ")");
  if (p.tmaps.empty()) return;
  bool changed = false;
  for (size_t i = 0; i < p.tmaps.size(); ++i) {
    const TmapSpec& t = p.tmaps[i];
    uint64_t addr = t.base.slot >= 0 ? v.h_argtab[t.base.slot] + (uint64_t)t.base.off : (uint64_t)t.base.off;
    if (addr == v.tmap_addr[i]) continue;
    encode_tmap_bf16(&v.h_tmaps[16 * i], (const void*)(uintptr_t)addr, t.inner, t.outer, t.row_bytes, t.box_inner,
                     t.box_outer);
    v.tmap_addr[i] = addr;
    changed = true;
  }
  // pageable source: staged by the driver before the call returns
  if (changed) CUDA_OK(cudaMemcpyAsync(v.d_tmaps, v.h_tmaps.data(), 128 * p.tmaps.size(), cudaMemcpyHostToDevice, s));
}

}  // namespace

namespace {

void launch_all(ExecVariant& v, cudaStream_t s) {
  for (const Launch& l : v.plan->launches) run_launch(l, v.d_argtab, s);
}

void launch_profiled(ExecVariant& v, cudaStream_t s) {
  ProfileState& ps = profile_state();
  std::vector<cudaEvent_t> evs(v.plan->launches.size() + 1);
  for (auto& e : evs) CUDA_OK(cudaEventCreate(&e));
  // the stream waits while the host enqueues, so events time kernels, not launch gaps
  launch_stream_hold(std::min<int64_t>(200000000, 20000 * (int64_t)v.plan->launches.size()), s);
  CUDA_OK(cudaEventRecord(evs[0], s));
  for (size_t i = 0; i < v.plan->launches.size(); ++i) {
    run_launch(v.plan->launches[i], v.d_argtab, s);
    CUDA_OK(cudaEventRecord(evs[i + 1], s));
  }
  CUDA_OK(cudaEventSynchronize(evs.back()));
  for (size_t i = 0; i < v.plan->launches.size(); ++i) {
    const Launch& l = v.plan->launches[i];
    float ms = 0;
    CUDA_OK(cudaEventElapsedTime(&ms, evs[i], evs[i + 1]));
    std::string key = std::string(kernel_kind_name(l.kind)) + "|" + l.label;
    ProfileEntry& e = ps.entries[key];
    e.kind = kernel_kind_name(l.kind);
    e.label = l.label;
    e.ms += ms;
    e.calls += 1;
    e.bytes += l.algo_bytes;
    e.flops += l.algo_flops;
  }
  for (auto& e : evs) cudaEventDestroy(e);
}

void run_variant(PJRT_Client* c, ExecVariant& v, cudaStream_t s) {
  const Plan& p = *v.plan;
  size_t dyn = (size_t)p.dyn_slots() * sizeof(uint64_t);
  // pageable source: the driver stages it before returning, so h_argtab can be reused
  if (dyn) CUDA_OK(cudaMemcpyAsync(v.d_argtab, v.h_argtab.data(), dyn, cudaMemcpyHostToDevice, s));
  refresh_tmaps(v, s);
  if (c->p2p) c->p2p->check();
  g_coll.comm = c->nccl_comm;
  g_coll.p2p = c->p2p;
  g_coll.ranks = c->opt.tp_size;
  g_coll.host_argtab = v.h_argtab.data();
  if (profile_state().enabled) {
    launch_profiled(v, s);
  } else if (c->opt.cuda_graphs && !v.graph_failed && v.runs >= 1) {
    if (!v.graph) {
      cudaGraph_t g = nullptr;
      CUDA_OK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      launch_all(v, s);
      cudaError_t e = cudaStreamEndCapture(s, &g);
      if (e != cudaSuccess || !g) {
        cudaGetLastError();
        v.graph_failed = true;
        launch_all(v, s);
      } else {
        v.graph_def = g;
        if (cudaGraphInstantiate(&v.graph, g, 0) != cudaSuccess) {
          cudaGetLastError();
          v.graph = nullptr;
          v.graph_failed = true;
          launch_all(v, s);
        }
      }
    }
    if (v.graph) {
      CUDA_OK(cudaGraphLaunch(v.graph, s));
      counters().graph_launches++;
    }
  } else {
    launch_all(v, s);
  }
  CUDA_OK(cudaGetLastError());
  if (v.status_host)  // checked at the next execution
    CUDA_OK(cudaMemcpyAsync(v.status_host, (char*)v.d_tmaps + 128 * p.tmaps.size(), sizeof(unsigned),
                            cudaMemcpyDeviceToHost, s));
  v.runs++;
  counters().executions++;
  counters().kernel_launches += (int64_t)p.launches.size();
}

}  // namespace

void exec_run(PJRT_LoadedExecutable* ex, PJRT_Buffer* const* args, size_t nargs, PJRT_Buffer** outs) {
  const Plan& p0 = *ex->copy.plan;
  PJRT_Client* c = ex->client;
  cudaStream_t s = c->stream;
  if (nargs != p0.params.size())
    fail(E_INVALID, "executable " + p0.name + " expects " + std::to_string(p0.params.size()) + " arguments, got " +
                        std::to_string(nargs));
  for (size_t i = 0; i < nargs; ++i) {
    PJRT_Buffer* b = args[i];
    if (!b) fail(E_INVALID, "null argument buffer " + std::to_string(i));
    const TensorSpec& t = p0.params[i];
    if (b->dt != t.dt || b->dims != t.shape)
      fail(E_INVALID, "argument " + std::to_string(i) + " has type " + dt_name(b->dt) + shape_str(b->dims) +
                          ", expected " + dt_name(t.dt) + shape_str(t.shape));
  }
  // a stale argument (an older version of an in-place updated buffer) is rebuilt first
  for (size_t i = 0; i < nargs; ++i) ensure_current(args[i]);
  // in place only when every updated argument is passed once and shares its storage with no other argument
  bool inplace = ex->inplace.plan != nullptr;
  if (inplace) {
    std::vector<const Storage*> st(nargs);
    for (size_t j = 0; j < nargs; ++j) st[j] = args[j]->ver->storage.get();
    std::sort(st.begin(), st.end());
    for (const InplaceDus& d : ex->inplace.plan->inplace) {
      const Storage* s0 = args[d.param]->ver->storage.get();
      const auto r = std::equal_range(st.begin(), st.end(), s0);
      if (r.second - r.first > 1) inplace = false;
    }
  }
  ExecVariant& v = inplace ? ex->inplace : ex->copy;
  const Plan& p = *v.plan;
  for (size_t i = 0; i < nargs; ++i) v.h_argtab[i] = (uint64_t)(uintptr_t)args[i]->ptr();
  std::vector<PJRT_Buffer*> created(p.outs.size(), nullptr);
  std::vector<std::shared_ptr<Version>> new_heads(p.inplace.size());
  std::vector<void*> undo(p.inplace.size(), nullptr);
  try {
    for (size_t k = 0; k < p.outs.size(); ++k) {
      if (p.out_alias_param[k] >= 0) continue;
      created[k] = new_buffer(c, p.outs[k].dt, p.outs[k].shape);
      v.h_argtab[p.params.size() + k] = (uint64_t)(uintptr_t)created[k]->ptr();
    }
    for (size_t u = 0; u < p.inplace.size(); ++u) {
      const InplaceDus& d = p.inplace[u];
      PJRT_Buffer* src = args[d.param];
      undo[u] = client_alloc(c, (size_t)d.undo_bytes);
      v.h_argtab[d.undo_slot] = (uint64_t)(uintptr_t)undo[u];
      v.h_argtab[p.params.size() + d.out] = (uint64_t)(uintptr_t)src->ptr();
      auto* b = new PJRT_Buffer();
      b->client = c;
      b->dt = p.outs[d.out].dt;
      b->dims = p.outs[d.out].shape;
      b->bytes = (size_t)p.outs[d.out].bytes();
      b->ver = std::make_shared<Version>();
      b->ver->storage = src->ver->storage;
      b->ver->client = c;
      created[d.out] = b;
      new_heads[u] = b->ver;
    }
  } catch (...) {
    for (auto* b : created) delete b;
    for (size_t u = 0; u < undo.size(); ++u) client_free(c, undo[u], (size_t)p.inplace[u].undo_bytes);
    throw;
  }
  run_variant(c, v, s);
  // the arguments updated in place become versions one behind their results
  for (size_t u = 0; u < p.inplace.size(); ++u) {
    const InplaceDus& d = p.inplace[u];
    Version* old = args[d.param]->ver.get();
    old->newer = new_heads[u];
    old->undo = undo[u];
    old->undo_bytes = (size_t)d.undo_bytes;
    old->rank = d.rank;
    old->dt = d.dt;
    for (int i = 0; i < d.rank; ++i) {
      old->out_shape[i] = d.out_shape[i];
      old->upd_shape[i] = d.upd_shape[i];
    }
  }
  for (size_t k = 0; k < created.size(); ++k) outs[k] = created[k];
}

}  // namespace cljxla
