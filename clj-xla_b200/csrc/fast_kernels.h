// Parameter blocks and entry points of the specialised kernels (decode GEMV,
// fused decode attention, ...), selected by the planner where a graph
// pattern allows and verified by the same host-side bounds checker.
#pragma once

#include <functional>

#include "planner.h"

namespace cljxla {

// Decode GEMV over up to GEMV_MAXSEG weight matrices that share the input x
// (the q / k / v projections of one layer, or gate / up): segment i covers
// rows [seg_end[i-1], seg_end[i]) of the launch, W_i is [N_i, K] row-major and
// y_i is [M, N_i].
constexpr int GEMV_MAXSEG = 4;
struct GemvParams {
  DPtr x;
  DPtr w[GEMV_MAXSEG], y[GEMV_MAXSEG];
  int64_t seg_end[GEMV_MAXSEG];
  int32_t y_dt[GEMV_MAXSEG];
  int32_t nseg, x_dt, w_dt, warps_per_row;
  int64_t M, N, K;  // N: rows of all segments
  int64_t x_sm;     // row stride (elements) of x
  // weights of the next GEMV in the schedule: each CTA, once its rows are done,
  // asks L2 for its share of them, so they stream in while the small kernels
  // between the two GEMVs run (byte counts are multiples of 16)
  DPtr pf[GEMV_MAXSEG];
  int64_t pf_bytes[GEMV_MAXSEG];
  int32_t npf;
  int32_t pro_out;  // K_GEMV_FUSED: the producer output that is x
  // K_GEMV_TAIL: arrival counter of the CTAs (zero between launches; the last
  // CTA to arrive runs the tail programs and resets it)
  DPtr tail_ctr;
  // the plan's status word (bounded waits of the bulk-copy GEMV report timeouts there)
  DPtr status;
  int32_t has_status, pad_s;
};

// Points every GEMV launch's prefetch at the weights of the next GEMV launch.
void link_gemv_prefetch(Plan& p);
// Points each staged decode attention's L2 hints at the weights of the GEMVs
// that follow it, up to a byte budget.
void link_attention_hints(Plan& p);

// Appends a GEMV whose x, M and K match the launch's as a further segment.
bool gemv_add_segment(Launch& l, const GemmParams& g);

using RegionFn = std::function<void(const DPtr&, int64_t, const char*)>;

// Tensor-core GEMM (k_gemm_tc.cu): C[M, N] = A[M, K] . B[N, K]^T, bf16
// operands with unit K stride, C dense row-major in c_dt (bf16 / f32).  The
// two tensor maps and the status word live in the executable's tensor-map
// table (Plan::tmaps); `a` / `b` / `a_ld` / `b_ld` tell the executor what to
// encode into them.
struct TcGemmParams {
  DPtr c, tmap_a, tmap_b, status;
  DPtr a, b;
  int64_t a_ld, b_ld;  // row strides in elements
  int32_t M, N, K, c_dt;
  int32_t tmap_a_index, tmap_b_index;
  // a_parts 3: A is an f32 matrix split exactly into three bf16 planes
  // (hi, mid, lo; plane p holds rows p * a_plane_rows ..), each multiplied by
  // the same B tile into one accumulator; a_parts 1: A is bf16
  int32_t a_parts, a_plane_rows;
  // tile width along N (256, or 64 for few rows of A: batched decode), rows of
  // A per copy (a multiple of 8, at most 128: only the rows a short A has), and
  // the K splits: with ksplit > 1 each (N tile, K split) unit stores its f32
  // partial tile in `part` ([ksplit][M][N]) and the last unit of an N tile to
  // arrive (counters: one per N tile, zero between launches) sums them in
  // split order, rounds and stores C
  int32_t bn, a_box, ksplit;
  // B is a graph parameter no launch writes (a weight): its first stages are
  // copied before the dependency wait
  int32_t b_const;
  DPtr part, counters;
};
// tile width and K splits for an M x N x K product on `sms` SMs
void tc_gemm_choose(int64_t M, int64_t N, int64_t K, int sms, int* bn, int* a_box, int* ksplit);

void launch_tc_gemm(const TcGemmParams& p, const uint64_t* argtab, cudaStream_t s);
bool make_tc_gemm(const GemmParams& g, TcGemmParams& out);
// f32 x bf16 product through three bf16 planes of the f32 operand (the caller
// supplies the planes as A; g.a_dt names the original f32 operand)
bool make_tc_gemm_split(const GemmParams& g, TcGemmParams& out);
void verify_tc_gemm(const TcGemmParams& p, const RegionFn& region);
void tc_gemm_tile_shape(int* bm, int* bn, int* bk);
// Encodes a 2-D bf16 tensor map (128-byte swizzle) into out128.
void encode_tmap_bf16(void* out128, const void* base, int64_t inner, int64_t outer, int64_t row_bytes, int box_inner,
                      int box_outer);

void launch_gemv(const GemvParams& p, const uint64_t* argtab, cudaStream_t s);
bool make_gemv(const GemmParams& g, Launch& out);
void verify_gemv(const Plan& plan, const Launch& l, const RegionFn& region);
void verify_fast_launch_impl(const Plan& p, const Launch& l, const RegionFn& region);

// Greedy-sampling argmax over the last axis (k_argmax.cu): in [..., V] float,
// out [rows] i32, the highest index among equal maxima (tensor.clj:519-532).
struct ArgmaxParams {
  TView in;
  DPtr out, part, counters;  // part / counters: ctas > 1 (a row split over CTAs)
  int64_t rows, V;
  int32_t ctas, pad;
};
void launch_argmax(const ArgmaxParams& p, const uint64_t* argtab, cudaStream_t s);
void verify_argmax(const ArgmaxParams& p, const RegionFn& region);
int64_t argmax_part_bytes(const ArgmaxParams& p);

}  // namespace cljxla

namespace cljxla {

// Fused attention (k_attention.cu).  q [B, nq, Sq, hd], k / v [B, nkv, T, hd],
// mask [B, nq, Sq, T] (broadcast view of the additive mask), out dense
// [B, nq, Sq, hd].  The printed score chain (scale / softcap, with its
// roundings) runs as a register program on each score.
constexpr int ATTN_MERGE_MAX_SPLITS = 64;  // position splits merged in-kernel (arrival counters)
constexpr int ATTN_MAX_HINTS = 4;          // weight regions a decode attention prefetches into L2

struct AttnParams {
  TView q, k, v, mask;
  DPtr out, part;
  // with position splits: one arrival counter per (batch*kv head, query tile),
  // zero between launches; the last split CTA to arrive merges the partials
  // itself and resets its counter (use_counters 0: a separate combine launch)
  DPtr counters;
  int32_t use_counters;
  int32_t use_tc;  // 1: decode on the tensor cores (64-position splits); 2: prefill on the tensor cores;
                   // 3: decode with bulk-copy staged K/V (one wave of CTAs, SIMT f32 arithmetic)
  int32_t B, nq, nkv, Sq, T, hd, group, splits, qtile;
  int32_t k_dt, dt_d1, dt_m, dt_sub, dt_exp, out_dt;
  int32_t nchain, chain_out;
  float mask_skip;
  // mask_mode 1: the additive mask is computed in the kernel, not read (the
  // planner proved it equal to the printed causal / sliding-window form, see
  // MaskForm): mask_mv where j - qpos > mask_gt or j - qpos < mask_lt, else
  // mask_z, with qpos = pos + qi + mask_off and pos the i32 at mask_pos when
  // has_mask_pos (else 0).  The mask view then has strides {0, 0, 1, 0}, so a
  // kernel's mask row offset is the query index qi.
  int32_t mask_mode, mask_gt, mask_lt, mask_off;
  float mask_mv, mask_z;
  DPtr mask_pos;
  int32_t has_mask_pos;
  // staged decode with a computed mask whose masked positions are skipped: the
  // splits share the live positions [qpos + mask_lt, qpos + mask_gt] evenly
  // instead of covering [0, T) in dec_per_split blocks
  int32_t dec_live_splits;
  EwInstr chain[12];
  // the chain in closed form where it is one (kernels skip the interpreter):
  // 0 general, 1 a multiply by chain_c rounded to chain_dt, 2 identity
  int32_t chain_kind;
  float chain_c;
  int32_t chain_dt, pad_k;
  // use_tc 3 (bulk-copy staged decode): positions per split and per staged chunk,
  // and the plan's status word, where a bounded wait that gives up is recorded
  int32_t dec_per_split, dec_chunk;
  DPtr status;
  int32_t has_status, pad_s;
  // weights of the GEMVs that follow, asked into L2 by this kernel's CTAs
  // before their dependency wait (the HBM is otherwise idle while a decode
  // attention runs); regions are 16-byte aligned multiples of 16 bytes
  DPtr hint[ATTN_MAX_HINTS];
  int64_t hint_bytes[ATTN_MAX_HINTS];
  int32_t nhint, pad_h;
};

void launch_attention(const AttnParams& p, const uint64_t* argtab, cudaStream_t s);
// whether the tensor-core decode kernel can run these views (bf16 q / K / V,
// 16-byte aligned rows, head_dim 64 / 128 / 256, one query tile of <= 8 vectors)
bool attention_tc_ok(const AttnParams& p);
// the bulk-copy staged decode kernel (Sq 1, bf16 K / V rows, 16-byte aligned),
// and its split / chunk sizes for one wave over `sms` SMs
bool attention_dec_ok(const AttnParams& p);
void plan_attention_dec(AttnParams& p, int sms);
// bytes of the per-split partial results an attention launch with splits > 1 needs
int64_t attention_part_bytes(const AttnParams& p);
// the tensor-core prefill kernel (64 query vectors per CTA, no position splits)
bool attention_tc_prefill_ok(const AttnParams& p);
void launch_attention_combine(const AttnParams& p, const uint64_t* argtab, cudaStream_t s);
void verify_attention(const Launch& l, const RegionFn& region);

// Pattern match of the printed attention block (attention.clj:343-365).
struct AttnMatch {
  int d2 = -1;          // probs . V dot (the node the fused kernel produces)
  int d1 = -1;          // q . K^T dot
  int q = -1, kc = -1, vc = -1;  // q [B,nq,Sq,hd]; K/V caches [B,nkv,T,hd] (before the GQA broadcast)
  int mask = -1;        // the mask operand of the add ([B,nq,Sq,T] view)
  int m = -1, sub = -1, exp = -1, div = -1;
  std::vector<int> chain;  // elementwise nodes from d1 to the mask add (exclusive), in order
  std::vector<int> absorbed;  // every node the fused kernel replaces (except d2)
  int group = 1;
};
// An attention mask operand proven equal to the causal / sliding-window form
// attention.clj:189-224 prints, either as the iota / compare / select chain of
// a traced position or as a dense literal: value mv where j - qpos > gt or
// (has_lt) j - qpos < lt, else z, with qpos = pos + qi + off and pos element 0
// of the i32 graph parameter pos_param (-1: none, pos = 0).
struct MaskForm {
  int pos_param = -1;
  int64_t off = 0, gt = 0, lt = 0;
  bool has_lt = false;
  float mv = 0.f, z = 0.f;
};
// Sq / T: the attention's query and key extents (axes 2 and 3 of the operand)
bool match_mask_form(const Graph& g, int mask, int64_t Sq, int64_t T, MaskForm& f);
std::vector<AttnMatch> match_attention(const Graph& g, const std::vector<char>& live,
                                       const std::vector<std::vector<int>>& users);

}  // namespace cljxla
