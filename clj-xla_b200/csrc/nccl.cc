// NCCL for tensor parallelism, loaded at run time (libnccl.so.2) so that a
// single-GPU user of the library needs no NCCL at all.  One communicator per
// client; the all_reduce(sum) of a plan is issued on the client's stream and
// is captured into the executable's CUDA graph like any kernel.
#include "nccl_rt.h"
#include "ir.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <mutex>

namespace cljxla {
namespace {

struct Nccl {
  decltype(&ncclGetUniqueId) get_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclGetErrorString) err = nullptr;
  bool ok = false;
};

Nccl& lib() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    // CLJXLA_B200_NCCL_LIB names the library to load instead (an NCCL outside
    // the loader path; tests point it at a missing file to make the load fail)
    void* h = nullptr;
    if (const char* path = getenv("CLJXLA_B200_NCCL_LIB")) {
      h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
    } else {
      h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
      if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    }
    if (!h) return;
    n.get_id = (decltype(n.get_id))dlsym(h, "ncclGetUniqueId");
    n.init_rank = (decltype(n.init_rank))dlsym(h, "ncclCommInitRank");
    n.all_reduce = (decltype(n.all_reduce))dlsym(h, "ncclAllReduce");
    n.destroy = (decltype(n.destroy))dlsym(h, "ncclCommDestroy");
    n.err = (decltype(n.err))dlsym(h, "ncclGetErrorString");
    n.ok = n.get_id && n.init_rank && n.all_reduce && n.destroy && n.err;
  });
  if (!n.ok) fail(E_PRECOND, "tensor parallelism needs NCCL (libnccl.so.2), which could not be loaded");
  return n;
}

void check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) fail(E_INTERNAL, std::string(what) + ": " + lib().err(r));
}

}  // namespace

std::string nccl_unique_id_hex() {
  ncclUniqueId id;
  check(lib().get_id(&id), "ncclGetUniqueId");
  static const char* hx = "0123456789abcdef";
  std::string s;
  for (size_t i = 0; i < sizeof(id.internal); ++i) {
    unsigned char c = (unsigned char)id.internal[i];
    s += hx[c >> 4];
    s += hx[c & 15];
  }
  return s;
}

void* nccl_comm_init(int nranks, int rank, const std::string& id_hex) {
  ncclUniqueId id;
  if (id_hex.size() != 2 * sizeof(id.internal)) fail(E_INVALID, "tp_nccl_id must be the hex form of an ncclUniqueId");
  auto val = [](char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    fail(E_INVALID, "tp_nccl_id is not hexadecimal");
  };
  for (size_t i = 0; i < sizeof(id.internal); ++i) id.internal[i] = (char)(val(id_hex[2 * i]) * 16 + val(id_hex[2 * i + 1]));
  ncclComm_t comm = nullptr;
  check(lib().init_rank(&comm, nranks, id, rank), "ncclCommInitRank");
  return (void*)comm;
}

void nccl_all_reduce(const void* src, void* dst, size_t count, int kdt, int reduce, void* comm, cudaStream_t s) {
  ncclDataType_t t;
  switch (kdt) {
    case KDT_F32: t = ncclFloat32; break;
    case KDT_BF16: t = ncclBfloat16; break;
    case KDT_F16: t = ncclFloat16; break;
    case KDT_I32: t = ncclInt32; break;
    default: fail(E_UNIMPLEMENTED, "all_reduce element type");
  }
  if (reduce != RED_ADD && reduce != RED_MAX) fail(E_UNIMPLEMENTED, "all_reduce reduction");
  check(lib().all_reduce(src, dst, count, t, reduce == RED_MAX ? ncclMax : ncclSum, (ncclComm_t)comm, s),
        "ncclAllReduce");
}

void nccl_comm_destroy(void* comm) {
  if (comm) lib().destroy((ncclComm_t)comm);
}

}  // namespace cljxla
