// Graph-level rewrites applied before planning.
//
// Common-subexpression elimination: the printed decoder graphs recompute
// identical values in every layer - the causal / sliding-window mask
// (attention.clj:192-217), the RoPE angle tables cos/sin(pos * freq)
// (attention.clj:29-44) and the dynamic-update-slice start-index conversions.
// Nodes with the same op, result type, attributes and (already canonical)
// operands are merged, so each such value is computed once per execution.
// Parameters are never merged; constants merge when their literals match.
#include <unordered_map>

#include "ir.h"

namespace cljxla {

namespace {

uint64_t mix(uint64_t h, uint64_t v) {
  h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
  return h;
}

uint64_t hash_vec(uint64_t h, const std::vector<int64_t>& v) {
  h = mix(h, v.size());
  for (auto x : v) h = mix(h, (uint64_t)x);
  return h;
}

bool same(const Node& a, const Node& b) {
  if (a.op != b.op || a.dt != b.dt || a.shape != b.shape || a.in != b.in || a.ia != b.ia || a.ib != b.ib ||
      a.ic != b.ic || a.id != b.id || a.i0 != b.i0 || a.splat != b.splat)
    return false;
  if (a.op == Op::Constant) {
    if (a.splat) return a.splat_val == b.splat_val || (a.splat_val != a.splat_val && b.splat_val != b.splat_val);
    return a.data == b.data;
  }
  return true;
}

}  // namespace

std::unique_ptr<Graph> cse_graph(const Graph& g, int* merged) {
  auto out = std::make_unique<Graph>();
  out->name = g.name;
  const int N = (int)g.nodes.size();
  std::vector<int> canon(N, -1);
  std::unordered_multimap<uint64_t, int> table;
  int nmerged = 0;
  for (int i = 0; i < N; ++i) {
    Node n = g.nodes[i];
    for (auto& x : n.in) x = canon[x];
    if (n.op != Op::Param) {
      uint64_t h = mix((uint64_t)n.op, (uint64_t)n.dt);
      h = hash_vec(h, n.shape);
      for (int x : n.in) h = mix(h, (uint64_t)x);
      h = hash_vec(hash_vec(hash_vec(hash_vec(h, n.ia), n.ib), n.ic), n.id);
      h = mix(h, (uint64_t)n.i0);
      if (n.op == Op::Constant) {
        if (n.splat) {
          uint64_t bits;
          memcpy(&bits, &n.splat_val, 8);
          h = mix(h, bits);
        } else {
          uint64_t dh = 1469598103934665603ull;
          for (uint8_t c : n.data) dh = (dh ^ c) * 1099511628211ull;
          h = mix(h, dh);
        }
      }
      bool found = false;
      auto range = table.equal_range(h);
      for (auto it = range.first; it != range.second; ++it) {
        if (same(out->nodes[it->second], n)) {
          canon[i] = it->second;
          found = true;
          break;
        }
      }
      if (found) {
        nmerged++;
        continue;
      }
      table.emplace(h, (int)out->nodes.size());
    }
    canon[i] = (int)out->nodes.size();
    out->nodes.push_back(std::move(n));
  }
  for (int p : g.params) out->params.push_back(canon[p]);
  for (int o : g.outputs) out->outputs.push_back(canon[o]);
  if (merged) *merged = nmerged;
  return out;
}

}  // namespace cljxla
