// The drop-in boundary: GetPjrtApi() and the PJRT entry points clj-xla's host
// calls (src/clj_xla/pjrt.clj).  Every entry returns a PJRT_Error* (NULL on
// success) and never aborts; C++ exceptions and CUDA errors become errors with
// the matching PJRT_Error_Code.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/cljxla_b200.h"
#include "jit.h"
#include "nccl_rt.h"
#include "runtime.h"

using namespace cljxla;

namespace {

PJRT_Error* make_error(int code, const std::string& msg) { return new PJRT_Error{code, msg}; }

template <class F>
PJRT_Error* guarded(F&& f) {
  try {
    f();
    return nullptr;
  } catch (const Error& e) {
    return make_error(e.code, e.what());
  } catch (const std::bad_alloc&) {
    return make_error(E_OOM, "host out of memory");
  } catch (const std::exception& e) {
    return make_error(E_INTERNAL, e.what());
  } catch (...) {
    return make_error(E_INTERNAL, "unknown error");
  }
}

template <class A>
A* args_of(void* p) {
  if (!p) fail(E_INVALID, "null argument struct");
  return (A*)p;
}

bool env_flag(const char* name, bool dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return !(v[0] == '0' || v[0] == 'f' || v[0] == 'F' || v[0] == 'n' || v[0] == 'N');
}

void set_device(PJRT_Client* c) { CUDA_OK(cudaSetDevice(c->device.ordinal)); }

// ------------------------------------------------------------------ errors
void Error_Destroy(void* a) {
  auto* args = (PJRT_Error_Destroy_Args*)a;
  if (args && args->error) delete args->error;
}

PJRT_Error* Error_Message(void* a) {
  auto* args = (PJRT_Error_Message_Args*)a;
  if (!args || !args->error) return nullptr;
  args->message = args->error->msg.c_str();
  args->message_size = args->error->msg.size();
  return nullptr;
}

PJRT_Error* Error_GetCode(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Error_GetCode_Args>(a);
    args->code = (PJRT_Error_Code)(args->error ? args->error->code : 0);
  });
}

PJRT_Error* Unimplemented(void*) {
  return make_error(E_UNIMPLEMENTED, "this PJRT entry point is not provided by libcljxla_b200");
}

// ------------------------------------------------------------------ plugin
PJRT_Error* Plugin_Initialize(void*) { return nullptr; }

PJRT_Error* Plugin_Attributes(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Plugin_Attributes_Args>(a);
    // one attribute: its array stride is then irrelevant to callers that
    // step by 56 (PJRT header) or by 64 bytes (pjrt.clj:131)
    static PJRT_NamedValue attr;
    static const char* k0 = "stablehlo_current_version";
    static const char* v0 = "1.0.0";
    attr.struct_size = sizeof(PJRT_NamedValue);
    attr.name = k0;
    attr.name_size = strlen(k0);
    attr.type = PJRT_NamedValue_kString;
    attr.string_value = v0;
    attr.value_size = strlen(v0);
    args->attributes = &attr;
    args->num_attributes = 1;
  });
}

// ------------------------------------------------------------------ events
PJRT_Event* new_event(PJRT_Client* c) {
  auto* e = new PJRT_Event();
  CUDA_OK(cudaEventCreateWithFlags(&e->ev, cudaEventDisableTiming));
  CUDA_OK(cudaEventRecord(e->ev, c->stream));
  return e;
}

PJRT_Error* Event_Destroy(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Event_Destroy_Args>(a);
    if (args->event) {
      if (args->event->ev) cudaEventDestroy(args->event->ev);
      delete args->event;
    }
  });
}

PJRT_Error* Event_IsReady(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Event_IsReady_Args>(a);
    if (!args->event) fail(E_INVALID, "null event");
    cudaError_t r = args->event->ev ? cudaEventQuery(args->event->ev) : cudaSuccess;
    args->is_ready = r != cudaErrorNotReady;
  });
}

PJRT_Error* Event_Await(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Event_Await_Args>(a);
    if (!args->event) fail(E_INVALID, "null event");
    if (args->event->ev) CUDA_OK(cudaEventSynchronize(args->event->ev));
    if (args->event->code) fail(args->event->code, args->event->msg);
  });
}

// ------------------------------------------------------------------ client
PJRT_Error* Client_Create(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Client_Create_Args>(a);
    auto c = std::make_unique<PJRT_Client>();
    ClientOptions& o = c->opt;
    o.fuse = env_flag("CLJXLA_B200_FUSE", true);
    o.fast_kernels = env_flag("CLJXLA_B200_FAST_KERNELS", true);
    o.cuda_graphs = env_flag("CLJXLA_B200_CUDA_GRAPHS", true);
    o.kv_in_place = env_flag("CLJXLA_B200_KV_IN_PLACE", true);
    if (const char* d = getenv("CLJXLA_B200_DEVICE")) o.device = atoi(d);
    if (const char* m = getenv("CLJXLA_B200_MEMORY_LIMIT")) o.memory_limit = atoll(m);
    size_t stride = sizeof(PJRT_NamedValue);
    if (args->num_options && args->create_options[0].struct_size >= sizeof(PJRT_NamedValue))
      stride = args->create_options[0].struct_size;  // clj-xla writes 64-byte elements
    for (size_t i = 0; i < args->num_options; ++i) {
      const PJRT_NamedValue& nv =
          *(const PJRT_NamedValue*)((const char*)args->create_options + i * stride);
      std::string k(nv.name, nv.name_size);
      auto as_bool = [&]() {
        if (nv.type == PJRT_NamedValue_kBool) return nv.bool_value;
        if (nv.type == PJRT_NamedValue_kInt64) return nv.int64_value != 0;
        if (nv.type == PJRT_NamedValue_kString) return std::string(nv.string_value, nv.value_size) == "true";
        return false;
      };
      if (k == "device" && nv.type == PJRT_NamedValue_kInt64) o.device = (int)nv.int64_value;
      else if (k == "fuse") o.fuse = as_bool();
      else if (k == "fast_kernels") o.fast_kernels = as_bool();
      else if (k == "cuda_graphs") o.cuda_graphs = as_bool();
      else if (k == "kv_in_place") o.kv_in_place = as_bool();
      else if (k == "tp_size" && nv.type == PJRT_NamedValue_kInt64) o.tp_size = (int)nv.int64_value;
      else if (k == "tp_rank" && nv.type == PJRT_NamedValue_kInt64) o.tp_rank = (int)nv.int64_value;
      else if (k == "tp_nccl_id" && nv.type == PJRT_NamedValue_kString) o.tp_nccl_id.assign(nv.string_value, nv.value_size);
      else if (k == "memory_limit_bytes" && nv.type == PJRT_NamedValue_kInt64) o.memory_limit = nv.int64_value;
      // other options (e.g. clj-xla's default {:allocator "platform"}) are accepted and ignored
    }
    if (o.tp_size < 1 || o.tp_rank < 0 || o.tp_rank >= o.tp_size) fail(E_INVALID, "bad tp_size / tp_rank");
    int ndev = 0;
    CUDA_OK(cudaGetDeviceCount(&ndev));
    if (ndev <= 0) fail(E_PRECOND, "no CUDA device visible");
    if (o.device < 0) {
      const char* lr = getenv("LOCAL_RANK");
      o.device = lr ? atoi(lr) % ndev : 0;
    }
    if (o.device >= ndev) fail(E_INVALID, "device ordinal out of range");
    c->device.ordinal = o.device;
    set_device(c.get());
    cudaDeviceProp prop;
    CUDA_OK(cudaGetDeviceProperties(&prop, o.device));
    if (prop.major < 10) fail(E_PRECOND, std::string("libcljxla_b200 needs an sm_100 device, found ") + prop.name);
    CUDA_OK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    cudaMemPool_t pool;
    CUDA_OK(cudaDeviceGetDefaultMemPool(&pool, o.device));
    uint64_t thresh = UINT64_MAX;
    CUDA_OK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thresh));
    if (o.tp_size > 1) {
      if (o.tp_nccl_id.empty()) fail(E_INVALID, "tp_size > 1 needs tp_nccl_id (cljxla_b200_nccl_unique_id on rank 0)");
      c->nccl_comm = nccl_comm_init(o.tp_size, o.tp_rank, o.tp_nccl_id);  // every rank joins here
    }
    args->client = c.release();
  });
}

PJRT_Error* Client_Destroy(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Client_Destroy_Args>(a);
    if (!args->client) return;
    set_device(args->client);
    cudaStreamSynchronize(args->client->stream);
    client_release_cached(args->client);
    cudaStreamSynchronize(args->client->stream);
    delete args->client->p2p;
    args->client->p2p = nullptr;
    nccl_comm_destroy(args->client->nccl_comm);
    cudaStreamDestroy(args->client->stream);
    if (args->client->pinned) cudaFreeHost(args->client->pinned);
    for (int i = 0; i < 2; ++i) {
      if (args->client->up_stage[i]) cudaFreeHost(args->client->up_stage[i]);
      if (args->client->up_done[i]) cudaEventDestroy(args->client->up_done[i]);
    }
    delete args->client;
  });
}

PJRT_Error* Client_PlatformName(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Client_PlatformName_Args>(a);
    if (!args->client) fail(E_INVALID, "null client");
    args->platform_name = args->client->platform.c_str();
    args->platform_name_size = args->client->platform.size();
  });
}

PJRT_Error* Client_AddressableDevices(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Client_AddressableDevices_Args>(a);
    if (!args->client) fail(E_INVALID, "null client");
    args->addressable_devices = args->client->device_list;
    args->num_addressable_devices = 1;  // one device facade (pjrt.clj:348-349)
  });
}

PJRT_Error* Client_Compile(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Client_Compile_Args>(a);
    PJRT_Client* c = args->client;
    if (!c || !args->program) fail(E_INVALID, "null client or program");
    const PJRT_Program* pr = args->program;
    std::string fmt(pr->format ? pr->format : "", pr->format ? pr->format_size : 0);
    if (fmt != "mlir") fail(E_INVALID, "unsupported program format '" + fmt + "' (expected mlir text)");
    std::lock_guard<std::mutex> lk(c->mu);
    set_device(c);
    auto graph = parse_mlir(pr->code, pr->code_size);
    PlanOptions po;
    po.fuse = c->opt.fuse;
    po.fast_kernels = c->opt.fast_kernels;
    po.kv_in_place = c->opt.kv_in_place;
    auto ex = std::make_unique<PJRT_LoadedExecutable>();
    ex->client = c;
    po.kv_in_place = false;
    ex->copy.plan = build_plan(*graph, po);
    if (c->opt.kv_in_place) {
      po.kv_in_place = true;
      auto ip = build_plan(*graph, po);
      if (!ip->inplace.empty()) ex->inplace.plan = std::move(ip);
    }
    prepare_jit(*ex->copy.plan);
    if (ex->inplace.plan) prepare_jit(*ex->inplace.plan);
    int64_t arena = ex->copy.plan->arena_bytes;
    if (ex->inplace.plan) arena = std::max(arena, ex->inplace.plan->arena_bytes);
    if (arena) {
      ex->arena = client_alloc(c, (size_t)arena);
      ex->arena_bytes = (size_t)arena;
      CUDA_OK(cudaStreamSynchronize(c->stream));  // the arena is used on other streams' schedules too
    }
    setup_variant(ex->copy, ex->arena);
    if (ex->inplace.plan) setup_variant(ex->inplace, ex->arena);
    args->executable = ex.release();
  });
}

// Uploads of at least this many bytes go through the client's pinned staging
// ring; smaller ones are one cudaMemcpyAsync from the caller's (pageable) memory.
constexpr size_t UPLOAD_STAGED_MIN = 8u << 20;
constexpr size_t UPLOAD_CHUNK = 32u << 20;

// Host-to-device copy of a large pageable host range (weight ingest,
// safetensors.clj:49-160 hands the plugin whole tensors): chunks of
// UPLOAD_CHUNK alternate between two pinned buffers; each chunk is copied into
// its buffer by several host threads in parallel (one thread's memcpy is well
// below the PCIe / C2C link rate) and then DMA'd on the client's stream, so the
// host copy of chunk i + 1 overlaps the DMA of chunk i.  Returns once the host
// data has been read; the DMAs complete in stream order.
static void upload_staged(PJRT_Client* c, void* dst, const void* src, size_t bytes) {
  for (int i = 0; i < 2; ++i) {
    if (!c->up_stage[i]) CUDA_OK(cudaMallocHost(&c->up_stage[i], UPLOAD_CHUNK));
    if (!c->up_done[i]) CUDA_OK(cudaEventCreateWithFlags(&c->up_done[i], cudaEventDisableTiming));
  }
  const unsigned hw = std::thread::hardware_concurrency();
  const int nthr = (int)std::max(1u, std::min(8u, hw ? hw : 1u));
  bool used[2] = {false, false};
  for (size_t off = 0, k = 0; off < bytes; off += UPLOAD_CHUNK, ++k) {
    const int b = (int)(k & 1);
    const size_t n = std::min(UPLOAD_CHUNK, bytes - off);
    if (used[b]) CUDA_OK(cudaEventSynchronize(c->up_done[b]));  // the DMA that last read this buffer
    char* stage = (char*)c->up_stage[b];
    const char* from = (const char*)src + off;
    const size_t piece = (n + nthr - 1) / nthr;
    std::vector<std::thread> th;
    for (int t = 1; t < nthr && (size_t)t * piece < n; ++t)
      th.emplace_back([=] { memcpy(stage + t * piece, from + t * piece, std::min(piece, n - t * piece)); });
    memcpy(stage, from, std::min(piece, n));
    for (auto& x : th) x.join();
    CUDA_OK(cudaMemcpyAsync((char*)dst + off, stage, n, cudaMemcpyHostToDevice, c->stream));
    CUDA_OK(cudaEventRecord(c->up_done[b], c->stream));
    used[b] = true;
  }
}

PJRT_Error* Client_BufferFromHostBuffer(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Client_BufferFromHostBuffer_Args>(a);
    PJRT_Client* c = args->client;
    if (!c) fail(E_INVALID, "null client");
    DT dt = dt_from_pjrt(args->type);
    if (dt == DT::INVALID) fail(E_UNIMPLEMENTED, "unsupported buffer element type " + std::to_string(args->type));
    std::vector<int64_t> dims(args->dims, args->dims + args->num_dims);
    for (auto d : dims)
      if (d < 0) fail(E_INVALID, "negative dimension");
    size_t es = dt_size(dt);
    size_t bytes = (size_t)numel(dims) * es;
    if (args->num_byte_strides) {  // only dense row-major host layouts are accepted
      int64_t expect = (int64_t)es;
      for (size_t i = args->num_dims; i-- > 0;) {
        if (args->byte_strides[i] != expect && dims[i] != 1)
          fail(E_UNIMPLEMENTED, "non-dense host byte_strides");
        expect *= dims[i];
      }
    }
    std::lock_guard<std::mutex> lk(c->mu);
    set_device(c);
    if (bytes && !args->data) fail(E_INVALID, "null host data");
    std::unique_ptr<PJRT_Buffer> b(new_buffer(c, dt, dims));
    if (bytes >= UPLOAD_STAGED_MIN) {
      upload_staged(c, b->ptr(), args->data, bytes);
      // the host buffer may be released once this event completes
      args->done_with_host_buffer = new_event(c);
    } else {
      // a host-to-device cudaMemcpyAsync from pageable memory copies the data
      // into the driver's staging memory before it returns: the host buffer is
      // free now, which a NULL event says (pjrt.clj:420-433 awaits only a
      // non-NULL one); from page-locked memory the copy reads it later
      bool pinned = false;
      if (bytes) {
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, args->data) == cudaSuccess) pinned = at.type == cudaMemoryTypeHost;
        cudaGetLastError();
        CUDA_OK(cudaMemcpyAsync(b->ptr(), args->data, bytes, cudaMemcpyHostToDevice, c->stream));
      }
      args->done_with_host_buffer = pinned ? new_event(c) : nullptr;
    }
    args->buffer = b.release();
  });
}

PJRT_Error* Buffer_Destroy(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Buffer_Destroy_Args>(a);
    PJRT_Buffer* b = args->buffer;
    if (!b) return;
    set_device(b->client);
    delete b;  // storage / undo records are released with their last version (stream ordered)
  });
}

PJRT_Error* Buffer_ElementType(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Buffer_ElementType_Args>(a);
    if (!args->buffer) fail(E_INVALID, "null buffer");
    args->type = (PJRT_Buffer_Type)dt_to_pjrt(args->buffer->dt);
  });
}

PJRT_Error* Buffer_Dimensions(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Buffer_Dimensions_Args>(a);
    if (!args->buffer) fail(E_INVALID, "null buffer");
    args->dims = args->buffer->dims.data();
    args->num_dims = args->buffer->dims.size();
  });
}

PJRT_Error* Buffer_OnDeviceSizeInBytes(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Buffer_OnDeviceSizeInBytes_Args>(a);
    if (!args->buffer) fail(E_INVALID, "null buffer");
    args->on_device_size_in_bytes = args->buffer->bytes;
  });
}

PJRT_Error* Buffer_ToHostBuffer(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Buffer_ToHostBuffer_Args>(a);
    PJRT_Buffer* b = args->src;
    if (!b) fail(E_INVALID, "null buffer");
    if (!args->dst) {
      args->dst_size = b->bytes;
      args->event = nullptr;
      return;
    }
    std::lock_guard<std::mutex> lk(b->client->mu);
    set_device(b->client);
    ensure_current(b);
    // the reference host always passes numel*4 bytes (pjrt.clj:535) and reads
    // what it needs; copy the buffer's bytes, never more than dst_size
    size_t n = std::min(b->bytes, args->dst_size);
    PJRT_Client* c = b->client;
    if (n >= (64u << 10)) {
      // large reads (decode logits): DMA into pinned staging, then one host copy;
      // a copy into pageable memory goes through the driver's smaller bounce buffer
      if (c->pinned_bytes < n) {
        if (c->pinned) CUDA_OK(cudaFreeHost(c->pinned));
        c->pinned = nullptr;
        c->pinned_bytes = 0;
        CUDA_OK(cudaMallocHost(&c->pinned, n));
        c->pinned_bytes = n;
      }
      CUDA_OK(cudaMemcpyAsync(c->pinned, b->ptr(), n, cudaMemcpyDeviceToHost, c->stream));
      CUDA_OK(cudaStreamSynchronize(c->stream));
      memcpy(args->dst, c->pinned, n);
    } else {
      if (n) CUDA_OK(cudaMemcpyAsync(args->dst, b->ptr(), n, cudaMemcpyDeviceToHost, c->stream));
      CUDA_OK(cudaStreamSynchronize(c->stream));
    }
    args->event = nullptr;
  });
}

// ------------------------------------------------------------- executables
PJRT_Error* LoadedExecutable_Destroy(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_LoadedExecutable_Destroy_Args>(a);
    PJRT_LoadedExecutable* ex = args->executable;
    if (!ex) return;
    set_device(ex->client);
    cudaStreamSynchronize(ex->client->stream);
    destroy_variant(ex->copy);
    destroy_variant(ex->inplace);
    if (ex->arena) {
      client_free(ex->client, ex->arena, ex->arena_bytes);
      cudaStreamSynchronize(ex->client->stream);
    }
    delete ex;
  });
}

PJRT_Error* Executable_NumOutputs(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_Executable_NumOutputs_Args>(a);
    if (!args->executable) fail(E_INVALID, "null executable");
    args->num_outputs = ((PJRT_LoadedExecutable*)args->executable)->copy.plan->outs.size();
  });
}

PJRT_Error* LoadedExecutable_Execute(void* a) {
  return guarded([&] {
    auto* args = args_of<PJRT_LoadedExecutable_Execute_Args>(a);
    PJRT_LoadedExecutable* ex = args->executable;
    if (!ex) fail(E_INVALID, "null executable");
    if (args->num_devices != 1) fail(E_INVALID, "libcljxla_b200 exposes exactly one addressable device");
    if (!args->argument_lists || !args->output_lists) fail(E_INVALID, "null argument or output lists");
    PJRT_Client* c = ex->client;
    std::lock_guard<std::mutex> lk(c->mu);
    set_device(c);
    exec_run(ex, args->argument_lists[0], args->num_args, args->output_lists[0]);
    if (args->device_complete_events) args->device_complete_events[0] = new_event(c);
  });
}

PJRT_Api make_api() {
  PJRT_Api api;
  memset(&api, 0, sizeof(api));
  api.struct_size = sizeof(PJRT_Api);
  api.pjrt_api_version.struct_size = sizeof(PJRT_Api_Version);
  api.pjrt_api_version.major_version = 0;
  api.pjrt_api_version.minor_version = 114;
  for (int i = 0; i < CLJXLA_PJRT_NUM_FNS; ++i) api.fns[i] = (void*)&Unimplemented;
  auto set = [&](int off, void* fn) { api.fns[(off - 40) / 8] = fn; };
  set(PJRT_OFF_ERROR_DESTROY, (void*)&Error_Destroy);
  set(PJRT_OFF_ERROR_MESSAGE, (void*)&Error_Message);
  set(PJRT_OFF_ERROR_GET_CODE, (void*)&Error_GetCode);
  set(PJRT_OFF_PLUGIN_INITIALIZE, (void*)&Plugin_Initialize);
  set(PJRT_OFF_PLUGIN_ATTRIBUTES, (void*)&Plugin_Attributes);
  set(PJRT_OFF_EVENT_DESTROY, (void*)&Event_Destroy);
  set(PJRT_OFF_EVENT_IS_READY, (void*)&Event_IsReady);
  set(PJRT_OFF_EVENT_AWAIT, (void*)&Event_Await);
  set(PJRT_OFF_CLIENT_CREATE, (void*)&Client_Create);
  set(PJRT_OFF_CLIENT_DESTROY, (void*)&Client_Destroy);
  set(PJRT_OFF_CLIENT_PLATFORM_NAME, (void*)&Client_PlatformName);
  set(PJRT_OFF_CLIENT_ADDRESSABLE_DEVICES, (void*)&Client_AddressableDevices);
  set(PJRT_OFF_CLIENT_COMPILE, (void*)&Client_Compile);
  set(PJRT_OFF_CLIENT_BUFFER_FROM_HOST_BUFFER, (void*)&Client_BufferFromHostBuffer);
  set(PJRT_OFF_EXECUTABLE_NUM_OUTPUTS, (void*)&Executable_NumOutputs);
  set(PJRT_OFF_LOADED_EXECUTABLE_DESTROY, (void*)&LoadedExecutable_Destroy);
  set(PJRT_OFF_LOADED_EXECUTABLE_EXECUTE, (void*)&LoadedExecutable_Execute);
  set(PJRT_OFF_BUFFER_DESTROY, (void*)&Buffer_Destroy);
  set(PJRT_OFF_BUFFER_ELEMENT_TYPE, (void*)&Buffer_ElementType);
  set(PJRT_OFF_BUFFER_DIMENSIONS, (void*)&Buffer_Dimensions);
  set(PJRT_OFF_BUFFER_ON_DEVICE_SIZE, (void*)&Buffer_OnDeviceSizeInBytes);
  set(PJRT_OFF_BUFFER_TO_HOST_BUFFER, (void*)&Buffer_ToHostBuffer);
  return api;
}

}  // namespace

extern "C" {

const PJRT_Api* GetPjrtApi(void) {
  static PJRT_Api api = make_api();
  return &api;
}

int64_t cljxla_b200_kernel_launches(void) { return counters().kernel_launches; }
int64_t cljxla_b200_executions(void) { return counters().executions; }

void cljxla_b200_profile_enable(int on) {
  profile_state().enabled = on != 0;
  if (on) profile_state().entries.clear();
}

size_t cljxla_b200_profile_dump(char* out, size_t cap) {
  std::string s = "[";
  bool first = true;
  for (auto& kv : profile_state().entries) {
    const ProfileEntry& e = kv.second;
    char buf[512];
    snprintf(buf, sizeof(buf), "%s{\"kind\":\"%s\",\"label\":\"%s\",\"ms\":%.6f,\"calls\":%lld,\"bytes\":%lld,\"flops\":%lld}",
             first ? "" : ",", e.kind.c_str(), e.label.c_str(), e.ms, (long long)e.calls, (long long)e.bytes,
             (long long)e.flops);
    s += buf;
    first = false;
  }
  s += "]";
  if (out && cap) {
    size_t n = std::min(cap - 1, s.size());
    memcpy(out, s.data(), n);
    out[n] = 0;
  }
  return s.size() + 1;
}

int cljxla_b200_plan_info(const PJRT_LoadedExecutable* ex, int64_t* info, int n) {
  if (!ex || !info) return -1;
  const Plan* pl = ex->inplace.plan ? ex->inplace.plan.get() : ex->copy.plan.get();  // the variant normally run
  int64_t v[8] = {(int64_t)pl->launches.size(), pl->arena_bytes, pl->n_nodes,
                  pl->n_live, pl->n_fused_groups, (int64_t)pl->const_blob.size(), pl->n_jit_missing,
                  pl->n_mask_computed};
  for (int i = 0; i < n && i < 8; ++i) info[i] = v[i];
  return 0;
}

void* cljxla_b200_stream(const PJRT_Client* c) { return c ? (void*)c->stream : nullptr; }

void* cljxla_b200_buffer_device_pointer(const PJRT_Buffer* b) { return b ? b->ptr() : nullptr; }

}  // extern "C"

extern "C" {

// Parses and plans MLIR text without touching a device (host-side checks).
// info[0..8) as cljxla_b200_plan_info (index 6, the kernels still to compile, is 0).  Returns 0, or the PJRT error code with
// the message copied into err.
CLJXLA_EXPORT int cljxla_b200_plan_text(const char* text, size_t len, int fuse, int64_t* info, int n, char* err,
                                        size_t errcap) {
  try {
    auto g = parse_mlir(text, len);
    PlanOptions po;
    po.fuse = (fuse & 1) != 0;        // bit 0: fusion
    po.kv_in_place = (fuse & 2) != 0;  // bit 1: in-place KV-cache updates
    auto p = build_plan(*g, po);
    int64_t v[8] = {(int64_t)p->launches.size(), p->arena_bytes, p->n_nodes, p->n_live, p->n_fused_groups,
                    (int64_t)p->const_blob.size(), 0, p->n_mask_computed};
    for (int i = 0; i < n && i < 8; ++i) info[i] = v[i];
    return 0;
  } catch (const Error& e) {
    if (err && errcap) snprintf(err, errcap, "%s", e.what());
    return e.code;
  } catch (const std::exception& e) {
    if (err && errcap) snprintf(err, errcap, "%s", e.what());
    return E_INTERNAL;
  }
}

CLJXLA_EXPORT int cljxla_b200_p2p_export(void* client, int64_t slot_bytes, char* out, size_t cap) {
  try {
    auto* c = (PJRT_Client*)client;
    if (!c || c->opt.tp_size < 2) return E_INVALID;
    std::lock_guard<std::mutex> lk(c->mu);
    set_device(c);
    if (!c->p2p) c->p2p = new P2PAllReduce();
    std::string h = c->p2p->export_handle(c->opt.tp_size, c->opt.tp_rank, slot_bytes);
    if (!out || cap < h.size() + 1) return E_INVALID;
    memcpy(out, h.c_str(), h.size() + 1);
    return 0;
  } catch (const Error& e) {
    return e.code;
  } catch (...) {
    return E_INTERNAL;
  }
}

CLJXLA_EXPORT int cljxla_b200_p2p_import(void* client, const char* handles, size_t len) {
  try {
    auto* c = (PJRT_Client*)client;
    if (!c || !c->p2p || !handles) return E_INVALID;
    std::lock_guard<std::mutex> lk(c->mu);
    set_device(c);
    c->p2p->import_handles(std::string(handles, len));
    return 0;
  } catch (const Error& e) {
    return e.code;
  } catch (...) {
    return E_INTERNAL;
  }
}

CLJXLA_EXPORT int cljxla_b200_nccl_unique_id(char* out, size_t cap) {
  try {
    std::string h = nccl_unique_id_hex();
    if (!out || cap < h.size() + 1) return E_INVALID;
    memcpy(out, h.c_str(), h.size() + 1);
    return 0;
  } catch (const Error& e) {
    return e.code;
  } catch (...) {
    return E_INTERNAL;
  }
}

CLJXLA_EXPORT void cljxla_b200_jit_cache_stats(int64_t* hits, int64_t* misses) { jit_disk_cache_stats(hits, misses); }

CLJXLA_EXPORT int cljxla_b200_jit_check(const char* text, size_t len, int flags, int* kernels, char* err,
                                        size_t errcap) {
  try {
    auto g = parse_mlir(text, len);
    PlanOptions po;
    po.fuse = (flags & 1) != 0;
    po.kv_in_place = (flags & 2) != 0;
    auto p = build_plan(*g, po);
    std::vector<std::string> src = jit_plan_sources(*p);
    if (kernels) *kernels = (int)src.size();
    std::string log;
    int failed = jit_check_sources(src, &log);
    if (failed > 0 && err && errcap) snprintf(err, errcap, "%s", log.c_str());
    return failed;
  } catch (const Error& e) {
    if (err && errcap) snprintf(err, errcap, "%s", e.what());
    return -2;
  } catch (const std::exception& e) {
    if (err && errcap) snprintf(err, errcap, "%s", e.what());
    return -2;
  }
}

}  // extern "C"
