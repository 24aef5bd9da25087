// Executes a launch plan: refresh the argument table, replay the captured
// CUDA graph (or launch eagerly the first time / when profiling).
#include <cuda_runtime.h>

#include <chrono>

#include "runtime.h"

namespace cljxla {

Counters& counters() {
  static Counters c;
  return c;
}

ProfileState& profile_state() {
  static ProfileState p;
  return p;
}

void run_launch(const Launch& l, const uint64_t* argtab, cudaStream_t s) {
  const void* b = l.blob.data();
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

namespace {

void launch_all(PJRT_LoadedExecutable* ex, cudaStream_t s) {
  for (const Launch& l : ex->plan->launches) run_launch(l, ex->d_argtab, s);
}

void launch_profiled(PJRT_LoadedExecutable* ex, cudaStream_t s) {
  ProfileState& ps = profile_state();
  std::vector<cudaEvent_t> evs(ex->plan->launches.size() + 1);
  for (auto& e : evs) CUDA_OK(cudaEventCreate(&e));
  CUDA_OK(cudaEventRecord(evs[0], s));
  for (size_t i = 0; i < ex->plan->launches.size(); ++i) {
    run_launch(ex->plan->launches[i], ex->d_argtab, s);
    CUDA_OK(cudaEventRecord(evs[i + 1], s));
  }
  CUDA_OK(cudaEventSynchronize(evs.back()));
  for (size_t i = 0; i < ex->plan->launches.size(); ++i) {
    const Launch& l = ex->plan->launches[i];
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

}  // namespace

void exec_run(PJRT_LoadedExecutable* ex, PJRT_Buffer* const* args, size_t nargs, PJRT_Buffer** outs) {
  Plan& p = *ex->plan;
  PJRT_Client* c = ex->client;
  cudaStream_t s = c->stream;
  if (nargs != p.params.size())
    fail(E_INVALID, "executable " + p.name + " expects " + std::to_string(p.params.size()) + " arguments, got " +
                        std::to_string(nargs));
  for (size_t i = 0; i < nargs; ++i) {
    PJRT_Buffer* b = args[i];
    if (!b) fail(E_INVALID, "null argument buffer " + std::to_string(i));
    const TensorSpec& t = p.params[i];
    if (b->dt != t.dt || b->dims != t.shape)
      fail(E_INVALID, "argument " + std::to_string(i) + " has type " + dt_name(b->dt) + shape_str(b->dims) +
                          ", expected " + dt_name(t.dt) + shape_str(t.shape));
    ex->h_argtab[i] = (uint64_t)(uintptr_t)b->ptr;
  }
  std::vector<PJRT_Buffer*> created;
  try {
    for (size_t k = 0; k < p.outs.size(); ++k) {
      auto* b = new PJRT_Buffer();
      created.push_back(b);
      b->client = c;
      b->dt = p.outs[k].dt;
      b->dims = p.outs[k].shape;
      b->bytes = (size_t)p.outs[k].bytes();
      if (b->bytes) CUDA_OK(cudaMallocAsync(&b->ptr, b->bytes, s));
      ex->h_argtab[p.params.size() + k] = (uint64_t)(uintptr_t)b->ptr;
    }
  } catch (...) {
    for (auto* b : created) {
      if (b->ptr) cudaFreeAsync(b->ptr, s);
      delete b;
    }
    throw;
  }
  // pageable source: the driver stages it before returning, so h_argtab can be reused
  size_t dyn = (p.params.size() + p.outs.size()) * sizeof(uint64_t);
  if (dyn) CUDA_OK(cudaMemcpyAsync(ex->d_argtab, ex->h_argtab.data(), dyn, cudaMemcpyHostToDevice, s));

  if (profile_state().enabled) {
    launch_profiled(ex, s);
  } else if (c->opt.cuda_graphs && !ex->graph_failed && ex->runs >= 1) {
    if (!ex->graph) {
      cudaGraph_t g = nullptr;
      CUDA_OK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      launch_all(ex, s);
      cudaError_t e = cudaStreamEndCapture(s, &g);
      if (e != cudaSuccess || !g) {
        cudaGetLastError();
        ex->graph_failed = true;
        launch_all(ex, s);
      } else {
        ex->graph_def = g;
        if (cudaGraphInstantiate(&ex->graph, g, 0) != cudaSuccess) {
          cudaGetLastError();
          ex->graph = nullptr;
          ex->graph_failed = true;
          launch_all(ex, s);
        }
      }
    }
    if (ex->graph) {
      CUDA_OK(cudaGraphLaunch(ex->graph, s));
      counters().graph_launches++;
    }
  } else {
    launch_all(ex, s);
  }
  CUDA_OK(cudaGetLastError());
  ex->runs++;
  counters().executions++;
  counters().kernel_launches += (int64_t)p.launches.size();
  for (size_t k = 0; k < created.size(); ++k) outs[k] = created[k];
}

}  // namespace cljxla
