// Decode attention with a fixed, statically allocated scratch.
//
// The split-KV attention kernel (k_attention.cu) writes per-split partial
// results (running max, sum and f32 context row) that attn_combine merges.
// Inside an executable those partials live in the executable's scratch arena,
// which Client_Compile allocates.  Some callers cannot allocate device memory
// at the point they want attention: a host that drives its own memory budget
// (a serving loop that has already handed all free HBM to a KV-cache pool), a
// caller inside an allocator callback, or code that must not trigger the
// stream-ordered pool's growth.  For them this entry point runs the same two
// kernels with the partials in a file-scope __device__ array of fixed size,
// so it allocates nothing: no cudaMalloc / cudaMallocAsync / cudaFree and no
// library routine that allocates.
//
// Limits and contract (also stated in include/cljxla_b200.h):
// * the scratch holds CLJXLA_STATIC_ATTN_SCRATCH_BYTES (1 MiB); a call whose
//   partials, splits * batch * q_heads * (head_dim + 2) * 4 bytes, exceed it
//   is rejected before anything is launched;
// * nothing in the scratch has to start at zero: every partial a combine
//   reads is written by the attention kernel of the same call first;
// * there is one scratch per device, so calls whose launches may overlap on
//   the device (different streams, or different host threads) race on it;
// * the first call on a device looks the scratch address up with
//   cudaGetSymbolAddress (which may load this module): make that first call
//   before any stream capture.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "fast_kernels.h"
#include "ir.h"
#include "../../include/cljxla_b200.h"

namespace cljxla {
namespace {

__device__ __align__(256) unsigned char g_static_attn_scratch[CLJXLA_STATIC_ATTN_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

int put_err(char* err, size_t cap, int code, const std::string& msg) {
  if (err && cap) {
    size_t n = msg.size() < cap - 1 ? msg.size() : cap - 1;
    memcpy(err, msg.data(), n);
    err[n] = 0;
  }
  return code;
}

TView dense4(const void* p, int dt, int64_t d0, int64_t d1, int64_t d2, int64_t d3) {
  TView v{};
  v.p.slot = -1;
  v.p.off = (int64_t)(uintptr_t)p;
  v.dt = dt;
  v.rank = 4;
  v.shape[0] = d0; v.shape[1] = d1; v.shape[2] = d2; v.shape[3] = d3;
  v.stride[3] = 1;
  v.stride[2] = d3;
  v.stride[1] = d2 * d3;
  v.stride[0] = d1 * d2 * d3;
  return v;
}

}  // namespace
}  // namespace cljxla

extern "C" CLJXLA_EXPORT int cljxla_b200_attention_decode_static(const void* q, const void* k_cache,
                                                                 const void* v_cache, const float* mask, void* out,
                                                                 int64_t batch, int64_t q_heads, int64_t kv_heads,
                                                                 int64_t positions, int64_t head_dim, float scale,
                                                                 void* stream, char* err, size_t errcap) {
  using namespace cljxla;
  if (!q || !k_cache || !v_cache || !mask || !out)
    return put_err(err, errcap, E_INVALID, "attention_decode_static: null pointer argument");
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || positions < 1)
    return put_err(err, errcap, E_INVALID, "attention_decode_static: sizes must be positive");
  if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256)
    return put_err(err, errcap, E_INVALID, "attention_decode_static: head_dim must be 32, 64, 128 or 256");
  if (q_heads % kv_heads != 0 || q_heads / kv_heads > 8)
    return put_err(err, errcap, E_INVALID,
                   "attention_decode_static: q_heads must be a multiple of kv_heads with at most 8 per KV head");
  if (batch * q_heads > (1 << 20) || batch * kv_heads > 65535 || positions > (1 << 24))
    return put_err(err, errcap, E_INVALID, "attention_decode_static: sizes out of range");
  const int64_t vec_bytes = head_dim / 32 * 2;  // each lane loads head_dim/32 bf16 values of a K/V row
  if ((uintptr_t)k_cache % vec_bytes || (uintptr_t)v_cache % vec_bytes)
    return put_err(err, errcap, E_INVALID, "attention_decode_static: K/V caches must be aligned to head_dim/16 bytes");

  // a failed launch inside surfaces as cljxla::Error; it must not cross the C ABI
  try {
    cudaGetLastError();  // a non-sticky error left by an earlier, unrelated call is not this call's failure
    AttnParams P{};
    P.B = (int32_t)batch;
    P.nq = (int32_t)q_heads;
    P.nkv = (int32_t)kv_heads;
    P.Sq = 1;
    P.T = (int32_t)positions;
    P.hd = (int32_t)head_dim;
    P.group = (int32_t)(q_heads / kv_heads);
    P.qtile = 1;
    P.q = dense4(q, KDT_BF16, batch, q_heads, 1, head_dim);
    P.k = dense4(k_cache, KDT_BF16, batch, kv_heads, positions, head_dim);
    P.v = dense4(v_cache, KDT_BF16, batch, kv_heads, positions, head_dim);
    P.mask = dense4(mask, KDT_F32, batch, q_heads, 1, positions);
    P.mask.stride[0] = P.mask.stride[1] = P.mask.stride[2] = 0;  // one additive row shared by all heads
    P.k_dt = KDT_BF16;
    // printed attention.clj:343-365 with a bf16 model: q.k^T rounded to bf16,
    // times the bf16 scale constant (rounded to bf16), + f32 mask, f32 softmax
    P.dt_d1 = KDT_BF16;
    P.dt_m = P.dt_sub = P.dt_exp = KDT_F32;
    P.out_dt = KDT_F32;
    P.mask_skip = -5000.0f;
    EwInstr imm{};
    imm.op = EW_IMM;
    imm.dt = (uint8_t)KDT_F32;
    imm.dst = 1;
    imm.fimm = bf16_to_f32(f32_to_bf16(scale));
    EwInstr mul{};
    mul.op = EW_MUL;
    mul.dt = (uint8_t)KDT_BF16;
    mul.a = 0;
    mul.b = 1;
    mul.dst = 2;
    P.chain[0] = imm;
    P.chain[1] = mul;
    P.nchain = 2;
    P.chain_out = 2;
    P.chain_kind = 1;  // the same multiply in closed form
    P.chain_c = imm.fimm;
    P.chain_dt = KDT_BF16;
    P.out.slot = -1;
    P.out.off = (int64_t)(uintptr_t)out;
    // same split rule as the planner: enough CTAs for two waves, >= 64 positions per split
    const int64_t ctas = batch * kv_heads;
    const int64_t sms = device_sm_count();
    int splits = 1;
    while (ctas * splits < 2 * sms && (int64_t)splits * 2 * 64 <= positions) splits *= 2;
    P.splits = splits;
    const int64_t part_bytes = (int64_t)splits * batch * q_heads * (head_dim + 2) * 4;
    if (splits > 1 && part_bytes > (int64_t)CLJXLA_STATIC_ATTN_SCRATCH_BYTES)
      return put_err(err, errcap, E_INVALID,
                     "attention_decode_static: partial results need " + std::to_string(part_bytes) +
                         " bytes, more than the static scratch of " +
                         std::to_string((long long)CLJXLA_STATIC_ATTN_SCRATCH_BYTES));
    if (splits > 1) {
      int dev = 0;
      cudaError_t e = cudaGetDevice(&dev);
      if (e != cudaSuccess) return put_err(err, errcap, E_INTERNAL, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
      if (dev < 0 || dev >= kMaxDevices) return put_err(err, errcap, E_INTERNAL, "device ordinal out of range");
      void* scratch = nullptr;
      {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
          e = cudaGetSymbolAddress(&g_scratch_addr[dev], g_static_attn_scratch);
          if (e != cudaSuccess) {
            g_scratch_addr[dev] = nullptr;
            return put_err(err, errcap, E_INTERNAL, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
          }
        }
        scratch = g_scratch_addr[dev];
      }
      P.part.slot = -1;
      P.part.off = (int64_t)(uintptr_t)scratch;
    }
    cudaStream_t s = (cudaStream_t)stream;
    launch_attention(P, nullptr, s);
    if (splits > 1) launch_attention_combine(P, nullptr, s);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return put_err(err, errcap, E_INTERNAL, std::string("launch: ") + cudaGetErrorString(e));
    return 0;
  } catch (const Error& e) {
    return put_err(err, errcap, e.code, std::string("attention_decode_static: ") + e.what());
  } catch (const std::exception& e) {
    return put_err(err, errcap, E_INTERNAL, std::string("attention_decode_static: ") + e.what());
  } catch (...) {
    return put_err(err, errcap, E_INTERNAL, "attention_decode_static: unknown failure");
  }
}
