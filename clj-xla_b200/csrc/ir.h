// In-memory form of a parsed StableHLO module (the subset printed by clj-xla's
// src/clj_xla/stablehlo.clj:248-600).
#pragma once

#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"

namespace cljxla {

enum class Op : uint8_t {
  Param, Constant,
  // elementwise
  Add, Sub, Mul, Div, Max, Min, Exp, Tanh, Sqrt, Rsqrt, Sin, Cos, Logistic, Neg, Abs,
  Convert, Compare, Select, Iota,
  // data movement
  Reshape, Transpose, Broadcast, Slice, Concat, DUS, Gather,
  // reductions / contractions
  Reduce, Dot,
  // collectives (tensor parallelism)
  AllReduce,
  // the NaN / Inf assertions of clj-xla's debug module (debug.clj:24-60), printed
  // as custom_call "check_non_nan" / "check_non_inf" (stablehlo.clj:562-570); i0:
  // 0 NaN, 1 Inf.  Their tensor<i1> result is never used by the printed graphs,
  // so they are dropped with the rest of the dead code.
  NanCheck,
};
const char* op_name(Op o);
inline bool op_is_elementwise(Op o) { return o >= Op::Add && o <= Op::Iota; }
inline bool op_is_unary_math(Op o) { return o >= Op::Exp && o <= Op::Abs; }

enum CmpDir : int { CMP_EQ = 0, CMP_NE, CMP_GE, CMP_GT, CMP_LE, CMP_LT };
enum ReduceKind : int { RED_ADD = 0, RED_MAX = 1 };

struct Node {
  Op op = Op::Param;
  DT dt = DT::F32;
  std::vector<int64_t> shape;
  std::vector<int> in;
  // op-specific attributes (see parser.cc for which op uses which list)
  std::vector<int64_t> ia, ib, ic, id;
  int64_t i0 = 0;
  // constants: either a splat value or packed element data of type dt
  bool splat = false;
  double splat_val = 0.0;
  std::vector<uint8_t> data;
  std::string name;
  int64_t numel() const { return cljxla::numel(shape); }
  int rank() const { return (int)shape.size(); }
};

struct Graph {
  std::string name;
  std::vector<Node> nodes;
  std::vector<int> params;   // node ids of func arguments, in order
  std::vector<int> outputs;  // node ids returned, in order
};

// Parses MLIR text; throws cljxla::Error (INVALID_ARGUMENT / UNIMPLEMENTED) on
// anything outside the supported subset.
std::unique_ptr<Graph> parse_mlir(const char* text, size_t len);

// Merges structurally identical nodes (common-subexpression elimination).
std::unique_ptr<Graph> cse_graph(const Graph& g, int* merged);

// Round-to-nearest-even conversions used for literals and host copies.
uint16_t f32_to_bf16(float f);
float bf16_to_f32(uint16_t b);
uint16_t f64_to_bf16(double d);
uint16_t f32_to_f16(float f);
float f16_to_f32(uint16_t h);

}  // namespace cljxla
