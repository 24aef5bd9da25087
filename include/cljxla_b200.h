/*
 * cljxla_b200.h - C ABI of libcljxla_b200.so, the B200 (sm_100a) executor
 * that clj-xla loads in place of its PJRT CPU plugin.
 *
 * The boundary is the PJRT C API.  clj-xla's host binds exactly one symbol,
 * GetPjrtApi (src/clj_xla/pjrt.clj:201-206 looks it up, :207 reads 984 bytes
 * of the returned table), and then calls these table slots: Error_Destroy /
 * Error_Message (pjrt.clj:63-82), Plugin_Initialize (:211-215),
 * Plugin_Attributes (:116-146), Event_Await / Event_Destroy (:420-433,
 * :508-522, :548-562), Client_Create (:261-275), Client_PlatformName
 * (:277-291), Client_AddressableDevices (:293-308), Client_Compile with format
 * "mlir" (:310-340), Client_BufferFromHostBuffer (:342-434),
 * LoadedExecutable_Execute (:454-525), Buffer_Destroy (:436-452) and
 * Buffer_ToHostBuffer (:527-611).  Struct layouts: pjrt_abi.h.
 *
 * The cljxla_b200_* functions are additions with no counterpart in the
 * reference; they expose counters and profiling for tests and benchmarks.
 */
#ifndef CLJXLA_B200_H_
#define CLJXLA_B200_H_

#include <stddef.h>
#include <stdint.h>

#include "pjrt_abi.h"

#if defined(__GNUC__)
#define CLJXLA_EXPORT __attribute__((visibility("default")))
#else
#define CLJXLA_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces the plugin entry point of xla_cpu_pjrt / jax_cuda12_pjrt that
 * clj-xla resolves at pjrt.clj:201-206. */
CLJXLA_EXPORT const PJRT_Api* GetPjrtApi(void);

/* Number of device kernels launched by executions so far (all executables). */
CLJXLA_EXPORT int64_t cljxla_b200_kernel_launches(void);

/* Number of LoadedExecutable_Execute calls completed so far. */
CLJXLA_EXPORT int64_t cljxla_b200_executions(void);

/* Per-kernel CUDA-event timing of subsequent executions (eager launches). */
CLJXLA_EXPORT void cljxla_b200_profile_enable(int on);

/* Writes the accumulated profile as JSON into out[cap]; returns the size needed. */
CLJXLA_EXPORT size_t cljxla_b200_profile_dump(char* out, size_t cap);

/* info[0..n): launches, scratch bytes, graph nodes, live nodes, fused
 * elementwise groups, constant bytes, launches whose compiled (NVRTC) form
 * failed so that an interpreting kernel runs instead, attention launches whose
 * causal / sliding-window mask is computed in the kernel instead of read.
 * Returns 0 on success. */
CLJXLA_EXPORT int cljxla_b200_plan_info(const PJRT_LoadedExecutable* exec, int64_t* info, int n);

/* Parses and plans MLIR text on the host only (no device needed).  `fuse`
 * holds flags: bit 0 enables fusion and the fast kernels, bit 1 plans
 * KV-cache updates in place.  info as above; returns 0 or a PJRT_Error_Code
 * with the message in err[errcap]. */
CLJXLA_EXPORT int cljxla_b200_plan_text(const char* text, size_t len, int fuse, int64_t* info, int n, char* err,
                                        size_t errcap);

/* Host-only check of the compiled fused kernels: plans the MLIR text (flags
 * as cljxla_b200_plan_text), generates the source of every fused elementwise
 * and row kernel and compiles each distinct one with NVRTC for sm_100a (no
 * device needed).  *kernels receives the number of generated kernels.
 * Returns the number that failed to compile (first log in err), -1 when
 * NVRTC is not available, -2 when planning failed. */
CLJXLA_EXPORT int cljxla_b200_jit_check(const char* text, size_t len, int flags, int* kernels, char* err,
                                        size_t errcap);

/* Programs this process found in (hits) or added to (misses) the on-disk
 * cache of compiled fused kernels.  The cache is keyed like clj-xla's compile
 * cache (src/clj_xla/compile.clj:13-24: SHA-256 of the program text), here of
 * each generated kernel's source with the NVRTC version and options, and
 * lives in CLJXLA_B200_CACHE_DIR (else $XDG_CACHE_HOME/cljxla_b200, else
 * $HOME/.cache/cljxla_b200; "0" turns it off).  No counterpart in the
 * reference, whose compile cache is in memory only. */
CLJXLA_EXPORT void cljxla_b200_jit_cache_stats(int64_t* hits, int64_t* misses);

/* Tensor parallelism (no counterpart in the reference, which runs on one
 * device).  A graph with "stablehlo.all_reduce" ops is one rank's shard of a
 * model; its client is created with the named values tp_size (int64),
 * tp_rank (int64) and tp_nccl_id (string): the hex id this function returns on
 * one rank (256 characters + NUL into out[cap]), passed to every rank by the
 * host.  Returns 0 or a PJRT_Error_Code (9: NCCL could not be loaded). */
CLJXLA_EXPORT int cljxla_b200_nccl_unique_id(char* out, size_t cap);

/* One-shot all-reduce over NVLink peer memory for tensor-parallel clients (no
 * counterpart in the reference).  Once every rank of a group has called
 * cljxla_b200_p2p_export (a CUDA IPC handle of a new exchange buffer with two
 * phases of one slot_bytes slot per rank, as hex: 128 characters + NUL into
 * out[cap]) and then cljxla_b200_p2p_import with all ranks' handles
 * concatenated in rank order, every all_reduce of at most slot_bytes (f32 or
 * bf16, 16-byte multiple) runs as one kernel per rank that stores its operand
 * into every rank's buffer, waits (bounded, about 16 s) for the others and
 * sums in rank order; larger ones stay on NCCL.  A wait that runs out makes
 * the client's next execution fail.  `client` is the PJRT_Client*. */
CLJXLA_EXPORT int cljxla_b200_p2p_export(void* client, int64_t slot_bytes, char* out, size_t cap);
CLJXLA_EXPORT int cljxla_b200_p2p_import(void* client, const char* handles, size_t len);

/* The cudaStream_t a client launches on (for event timing by the caller). */
CLJXLA_EXPORT void* cljxla_b200_stream(const PJRT_Client* client);

/* Device address backing a buffer. */
CLJXLA_EXPORT void* cljxla_b200_buffer_device_pointer(const PJRT_Buffer* buffer);

/* Size of the fixed device scratch used by cljxla_b200_attention_decode_static. */
#define CLJXLA_STATIC_ATTN_SCRATCH_BYTES (1u << 20)

/* Decode attention of one layer that allocates no device memory.  No
 * counterpart in the reference: it is the split-KV kernel an executable uses
 * for the printed attention block (attention.clj:343-365), callable directly
 * by hosts that cannot allocate at that point (all free memory already handed
 * to a KV pool, allocator callbacks, code that must not grow the memory pool).
 *
 *   q        bf16 [batch, q_heads, 1, head_dim]          (device)
 *   k_cache  bf16 [batch, kv_heads, positions, head_dim] (device, head_dim/16-byte aligned)
 *   v_cache  bf16 [batch, kv_heads, positions, head_dim] (device, same alignment)
 *   mask     f32  [positions] additive mask shared by every batch row and head (device)
 *   out      f32  [batch, q_heads, 1, head_dim]          (device)
 *
 * scores = bf16(bf16(q.k) * bf16(scale)) + mask, softmax in f32, out = p.v:
 * the printed graph's op order and roundings.  A position whose mask value is
 * at or below -5000 is skipped: it contributes weight 0, which is what the
 * formula gives for the -10000 causal mask whenever some position of the row
 * is unmasked.  A row whose every position is at or below -5000 therefore
 * yields zeros (the formula would give the uniform average, or NaN for -inf).
 * Failures (bad sizes, a failed launch) are returned, never thrown.  head_dim in {32,64,128,256},
 * q_heads a multiple of kv_heads with at most 8 per KV head.  Work is enqueued
 * on `stream` (a cudaStream_t; NULL = legacy default stream) of the calling
 * thread's current device.
 *
 * Partial results live in one file-scope device array per device of
 * CLJXLA_STATIC_ATTN_SCRATCH_BYTES; calls needing more
 * (splits * batch * q_heads * (head_dim + 2) * 4 bytes) are rejected before
 * anything runs.  Nothing in it has to start at zero.  Calls that may overlap
 * on the device race on the scratch.  The first call on each device looks up
 * the scratch address (and may load the module): make it before any stream
 * capture.  Returns 0, or a PJRT_Error_Code with the message in err[errcap]. */
CLJXLA_EXPORT int cljxla_b200_attention_decode_static(const void* q, const void* k_cache, const void* v_cache,
                                                      const float* mask, void* out, int64_t batch, int64_t q_heads,
                                                      int64_t kv_heads, int64_t positions, int64_t head_dim,
                                                      float scale, void* stream, char* err, size_t errcap);

#ifdef __cplusplus
}
#endif

#endif /* CLJXLA_B200_H_ */
