// Parser for the StableHLO text produced by clj-xla's printer
// (src/clj_xla/stablehlo.clj:248-600).  The grammar is small and regular:
//
//   module @name {
//     func.func @main(%a: tensor<..>, ...) -> (tensor<..>, ...) {
//       %v = stablehlo.constant dense<LIT> : T            (:269-270)
//       %v_1d = stablehlo.constant dense<[..]> : T1d      (:259-268, then a reshape)
//       %v = stablehlo.<op> %a, %b : T  [loc("..")]       (:577-579)
//       %v = stablehlo.reshape %a : (T) -> T              (:318-322)
//       %v = "stablehlo.<op>"(%a, ..) {attrs} : (Ts) -> T (convert/compare/select/gather/
//                                                          transpose/broadcast_in_dim/slice/
//                                                          dynamic_update_slice/iota/
//                                                          concatenate/dot_general)
//       %v_red = "stablehlo.reduce"(%a, %init) ({ ^bb0 .. region .. }) {dimensions = ..} : ..
//       return %a, .. : T, ..
//     }
//   }
//
// Literals can be hundreds of MB (static causal masks / RoPE tables), so the
// scanner works on the caller's buffer without copying lines.
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <string>
#include <string_view>
#include <thread>
#include <vector>

#include "ir.h"

namespace cljxla {

using sv = std::string_view;

const char* op_name(Op o) {
  static const char* names[] = {"param", "constant", "add", "subtract", "multiply", "divide", "maximum",
                                "minimum", "exponential", "tanh", "sqrt", "rsqrt", "sine", "cosine",
                                "logistic", "negate", "abs", "convert", "compare", "select", "iota",
                                "reshape", "transpose", "broadcast_in_dim", "slice", "concatenate",
                                "dynamic_update_slice", "gather", "reduce", "dot_general", "all_reduce",
                                "custom_call"};
  return names[(int)o];
}

uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;  // NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
uint16_t f64_to_bf16(double d) {
  // correctly rounded double -> bf16: pick the nearest of the bf16 neighbours
  // of the f32 rounding (avoids double rounding through f32)
  if (std::isnan(d)) return 0x7fc0;
  uint16_t c = f32_to_bf16((float)d);
  uint16_t best = c;
  double be = std::fabs(d - (double)bf16_to_f32(c));
  for (int k = -1; k <= 1; k += 2) {
    uint16_t n = (uint16_t)(c + k);
    float nf = bf16_to_f32(n);
    if (std::isnan(nf)) continue;
    double e = std::fabs(d - (double)nf);
    if (e < be || (e == be && (n & 1) == 0)) { best = n; be = e; }
  }
  return best;
}
uint16_t f32_to_f16(float f) {
  // IEEE binary16, round to nearest even (host-side literal conversion only)
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  uint32_t mant = x & 0x7fffffu;
  if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0));
  if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - exp);
    uint32_t half = 1u << (shift - 1);
    uint32_t r = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1);
    if (rem > half || (rem == half && (r & 1))) r++;
    return (uint16_t)(sign | r);
  }
  uint32_t r = mant >> 13;
  uint32_t rem = mant & 0x1fffu;
  uint32_t out = sign | ((uint32_t)exp << 10) | r;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) out++;
  return (uint16_t)out;
}
float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ffu;
  uint32_t u;
  if (exp == 0) {
    if (mant == 0) {
      u = sign;
    } else {
      int e = -1;
      do { e++; mant <<= 1; } while (!(mant & 0x400u));
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (mant << 13);
  } else {
    u = sign | ((exp - 15 + 127) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

namespace {

[[noreturn]] void perr(const std::string& m, sv line) {
  std::string l(line.substr(0, 200));
  fail(E_INVALID, "MLIR parse error: " + m + " in line: " + l);
}

inline sv trim(sv s) {
  while (!s.empty() && (s.front() == ' ' || s.front() == '\t' || s.front() == '\r')) s.remove_prefix(1);
  while (!s.empty() && (s.back() == ' ' || s.back() == '\t' || s.back() == '\r')) s.remove_suffix(1);
  return s;
}
inline bool starts(sv s, sv p) { return s.size() >= p.size() && s.substr(0, p.size()) == p; }

struct Type {
  std::vector<int64_t> shape;
  DT dt = DT::INVALID;
};

Type parse_type(sv s, sv line) {
  s = trim(s);
  if (!starts(s, "tensor<") || s.back() != '>') perr("bad tensor type '" + std::string(s) + "'", line);
  sv body = s.substr(7, s.size() - 8);
  Type t;
  size_t pos = 0;
  while (true) {
    size_t x = body.find('x', pos);
    if (x == sv::npos) break;
    sv part = body.substr(pos, x - pos);
    if (part.empty() || !(part[0] >= '0' && part[0] <= '9')) break;
    int64_t v = 0;
    for (char c : part) {
      if (c < '0' || c > '9') perr("bad dim", line);
      v = v * 10 + (c - '0');
    }
    t.shape.push_back(v);
    pos = x + 1;
  }
  t.dt = dt_from_name(std::string(body.substr(pos)));
  if (t.dt == DT::INVALID) perr("unsupported element type '" + std::string(body.substr(pos)) + "'", line);
  return t;
}

// Finds "key = " where key is not preceded by an identifier character.
size_t find_key(sv s, sv key) {
  size_t p = 0;
  while ((p = s.find(key, p)) != sv::npos) {
    bool ok_before = p == 0 || !(isalnum((unsigned char)s[p - 1]) || s[p - 1] == '_');
    size_t e = p + key.size();
    if (ok_before && s.substr(e, 3) == " = ") return e + 3;
    p = e;
  }
  return sv::npos;
}

std::vector<int64_t> parse_int_list_at(sv s, size_t p, sv line) {
  // accepts "array<i64: a, b>", "array<i64>", "[a, b]", "[]"
  std::vector<int64_t> out;
  sv r = s.substr(p);
  size_t end;
  if (starts(r, "array<i64>")) return out;
  if (starts(r, "array<i64:")) {
    end = r.find('>');
    r = r.substr(10, end - 10);
  } else if (starts(r, "[")) {
    end = r.find(']');
    r = r.substr(1, end - 1);
  } else {
    perr("expected integer list", line);
  }
  const char* c = r.data();
  const char* e = c + r.size();
  while (c < e) {
    while (c < e && (*c == ' ' || *c == ',')) c++;
    if (c >= e) break;
    char* nx;
    long long v = strtoll(c, &nx, 10);
    if (nx == c) perr("bad integer in list", line);
    out.push_back(v);
    c = nx;
  }
  return out;
}

std::vector<int64_t> attr_list(sv attrs, sv key, sv line, bool required = true) {
  size_t p = find_key(attrs, key);
  if (p == sv::npos) {
    if (required) perr("missing attribute " + std::string(key), line);
    return {};
  }
  return parse_int_list_at(attrs, p, line);
}
int64_t attr_int(sv attrs, sv key, sv line) {
  size_t p = find_key(attrs, key);
  if (p == sv::npos) perr("missing attribute " + std::string(key), line);
  return strtoll(attrs.data() + p, nullptr, 10);
}

// splits "%a, %b, %c" (top level) into names
std::vector<std::string> parse_operands(sv s, sv line) {
  std::vector<std::string> out;
  size_t i = 0;
  while (i < s.size()) {
    while (i < s.size() && (s[i] == ' ' || s[i] == ',')) i++;
    if (i >= s.size()) break;
    if (s[i] != '%') perr("expected operand", line);
    size_t j = i + 1;
    while (j < s.size() && s[j] != ',' && s[j] != ' ' && s[j] != ')') j++;
    out.emplace_back(s.substr(i + 1, j - i - 1));
    i = j;
  }
  return out;
}

// splits a comma separated list of types at top level (types contain no commas)
std::vector<Type> parse_type_list(sv s, sv line) {
  std::vector<Type> out;
  size_t i = 0;
  while (i < s.size()) {
    size_t j = s.find(',', i);
    if (j == sv::npos) j = s.size();
    sv t = trim(s.substr(i, j - i));
    if (!t.empty()) out.push_back(parse_type(t, line));
    i = j + 1;
  }
  return out;
}

void store_literal(Node& n, const std::vector<double>& vals) {
  size_t cnt = vals.size();
  n.data.resize(cnt * dt_size(n.dt));
  uint8_t* p = n.data.data();
  for (size_t i = 0; i < cnt; ++i) {
    double v = vals[i];
    switch (n.dt) {
      case DT::F32: { float f = (float)v; memcpy(p + 4 * i, &f, 4); break; }
      case DT::BF16: { uint16_t b = f64_to_bf16(v); memcpy(p + 2 * i, &b, 2); break; }
      case DT::F16: { uint16_t h = f32_to_f16((float)v); memcpy(p + 2 * i, &h, 2); break; }
      case DT::F64: memcpy(p + 8 * i, &v, 8); break;
      case DT::I32: case DT::U32: { int32_t x = (int32_t)(int64_t)v; memcpy(p + 4 * i, &x, 4); break; }
      case DT::I64: { int64_t x = (int64_t)v; memcpy(p + 8 * i, &x, 8); break; }
      case DT::I16: { int16_t x = (int16_t)(int64_t)v; memcpy(p + 2 * i, &x, 2); break; }
      case DT::I8: case DT::U8: case DT::I1: { int8_t x = (int8_t)(int64_t)v; p[i] = (uint8_t)x; break; }
      default: fail(E_UNIMPLEMENTED, "literal of unsupported type");
    }
  }
}

double round_to_dt(double v, DT dt) {
  switch (dt) {
    case DT::F32: return (double)(float)v;
    case DT::BF16: return (double)bf16_to_f32(f64_to_bf16(v));
    case DT::F16: return (double)f16_to_f32(f32_to_f16((float)v));
    case DT::F64: return v;
    case DT::I1: return v != 0 ? 1.0 : 0.0;
    default: return std::trunc(v);
  }
}

// Decimal numbers of up to 15 significant digits and a power of ten within
// 10^+-22 (every value the printer writes with %.6e, stablehlo.clj:269-270,
// and every integer literal) convert exactly: the digits form an integer
// below 2^53 and both it and the power of ten are exact doubles, so one
// multiplication or division rounds once, as strtod does (Clinger's fast
// path).  Anything else (more digits, larger exponents, inf / nan) goes to
// strtod.  Returns false when the token is not a number of this form.
bool fast_decimal(const char*& c, const char* e, double* out) {
  static const double kPow10[23] = {1e0,  1e1,  1e2,  1e3,  1e4,  1e5,  1e6,  1e7,  1e8,  1e9,  1e10, 1e11,
                                    1e12, 1e13, 1e14, 1e15, 1e16, 1e17, 1e18, 1e19, 1e20, 1e21, 1e22};
  const char* p = c;
  bool neg = false;
  if (p < e && (*p == '-' || *p == '+')) neg = *p++ == '-';
  uint64_t m = 0;
  int digits = 0, frac = 0;
  bool any = false;
  while (p < e && *p >= '0' && *p <= '9') {
    if (m || *p != '0') ++digits;
    m = m * 10 + (uint64_t)(*p++ - '0');
    any = true;
    if (digits > 15) return false;
  }
  if (p < e && *p == '.') {
    ++p;
    while (p < e && *p >= '0' && *p <= '9') {
      if (m || *p != '0') ++digits;
      m = m * 10 + (uint64_t)(*p++ - '0');
      ++frac;
      any = true;
      if (digits > 15) return false;
    }
  }
  if (!any) return false;
  int ex = 0;
  if (p < e && (*p == 'e' || *p == 'E')) {
    ++p;
    bool eneg = false;
    if (p < e && (*p == '-' || *p == '+')) eneg = *p++ == '-';
    if (p >= e || *p < '0' || *p > '9') return false;
    while (p < e && *p >= '0' && *p <= '9') {
      ex = ex * 10 + (*p++ - '0');
      if (ex > 400) return false;
    }
    if (eneg) ex = -ex;
  }
  if (p < e && ((*p >= 'a' && *p <= 'z') || (*p >= 'A' && *p <= 'Z'))) return false;  // e.g. "inf"
  const int k = ex - frac;
  double v = (double)m;
  if (k < -22 || k > 22) return false;
  v = k < 0 ? v / kPow10[-k] : v * kPow10[k];
  *out = neg ? -v : v;
  c = p;
  return true;
}

double parse_scalar_token(const char*& c, const char* e, sv line) {
  while (c < e && *c == ' ') c++;
  if (e - c >= 4 && !memcmp(c, "true", 4)) { c += 4; return 1.0; }
  if (e - c >= 5 && !memcmp(c, "false", 5)) { c += 5; return 0.0; }
  double v;
  if (fast_decimal(c, e, &v)) return v;
  char* nx;
  v = strtod(c, &nx);
  if (nx == c) perr("bad literal value", line);
  c = nx;
  return v;
}

// the comma-separated values between c and e (no brackets) into vals, in order
void parse_values(const char* c, const char* e, std::vector<double>& vals, sv line) {
  while (c < e) {
    while (c < e && (*c == ' ' || *c == ',' || *c == '[' || *c == ']')) c++;
    if (c >= e) break;
    vals.push_back(parse_scalar_token(c, e, line));
  }
}

}  // namespace

DT dt_from_name(const std::string& s) {
  if (s == "f32") return DT::F32;
  if (s == "bf16") return DT::BF16;
  if (s == "f16") return DT::F16;
  if (s == "f64") return DT::F64;
  if (s == "i32" || s == "si32") return DT::I32;
  if (s == "i64") return DT::I64;
  if (s == "i8") return DT::I8;
  if (s == "i16") return DT::I16;
  if (s == "ui8" || s == "u8") return DT::U8;
  if (s == "ui32" || s == "u32") return DT::U32;
  if (s == "i1") return DT::I1;
  return DT::INVALID;
}
const char* dt_name(DT t) {
  switch (t) {
    case DT::F32: return "f32";
    case DT::BF16: return "bf16";
    case DT::F16: return "f16";
    case DT::F64: return "f64";
    case DT::I32: return "i32";
    case DT::I64: return "i64";
    case DT::I8: return "i8";
    case DT::I16: return "i16";
    case DT::U8: return "ui8";
    case DT::U32: return "ui32";
    case DT::I1: return "i1";
    default: return "invalid";
  }
}
DT dt_from_pjrt(int t) {
  switch (t) {
    case 1: return DT::I1;
    case 2: return DT::I8;
    case 3: return DT::I16;
    case 4: return DT::I32;
    case 5: return DT::I64;
    case 6: return DT::U8;
    case 8: return DT::U32;
    case 10: return DT::F16;
    case 11: return DT::F32;
    case 12: return DT::F64;
    case 13: return DT::BF16;
    default: return DT::INVALID;
  }
}
int dt_to_pjrt(DT t) {
  switch (t) {
    case DT::I1: return 1;
    case DT::I8: return 2;
    case DT::I16: return 3;
    case DT::I32: return 4;
    case DT::I64: return 5;
    case DT::U8: return 6;
    case DT::U32: return 8;
    case DT::F16: return 10;
    case DT::F32: return 11;
    case DT::F64: return 12;
    case DT::BF16: return 13;
    default: return 0;
  }
}
std::string shape_str(const std::vector<int64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) o += (i ? "," : "") + std::to_string(s[i]);
  return o + "]";
}
void fail(int code, const std::string& msg) { throw Error(code, msg); }

std::unique_ptr<Graph> parse_mlir(const char* text, size_t len) {
  auto g = std::make_unique<Graph>();
  std::unordered_map<std::string, int> ids;
  bool in_func = false, have_return = false;

  auto lookup = [&](const std::string& n, sv line) -> int {
    auto it = ids.find(n);
    if (it == ids.end()) perr("undefined value %" + n, line);
    return it->second;
  };
  auto add_node = [&](Node&& n, sv line) -> int {
    if (ids.count(n.name)) perr("redefinition of %" + n.name, line);
    int id = (int)g->nodes.size();
    ids[n.name] = id;
    g->nodes.push_back(std::move(n));
    return id;
  };

  const char* p = text;
  const char* end = text + len;
  while (p < end) {
    const char* nl = (const char*)memchr(p, '\n', (size_t)(end - p));
    if (!nl) nl = end;
    sv raw(p, (size_t)(nl - p));
    p = nl + 1;
    sv line = trim(raw);
    if (line.empty() || line == "}") continue;
    // strip a trailing loc("...") (stablehlo.clj:552-553)
    if (line.back() == ')') {
      size_t lp = line.rfind(" loc(\"");
      if (lp != sv::npos) line = trim(line.substr(0, lp));
    }
    if (starts(line, "module @")) {
      sv nm = line.substr(8);
      size_t sp = nm.find_first_of(" {");
      g->name = std::string(nm.substr(0, sp));
      continue;
    }
    if (starts(line, "func.func @main(")) {
      if (in_func) perr("nested function", line);
      in_func = true;
      sv sig = line.substr(16);
      size_t close = sig.find(") -> ");
      if (close == sv::npos) perr("bad function signature", line);
      sv params = sig.substr(0, close);
      size_t i = 0;
      while (i < params.size()) {
        size_t comma = params.find(", %", i);
        sv one = params.substr(i, comma == sv::npos ? sv::npos : comma - i);
        size_t colon = one.find(':');
        if (one.empty() || one[0] != '%' || colon == sv::npos) perr("bad parameter", line);
        Node n;
        n.op = Op::Param;
        n.name = std::string(one.substr(1, colon - 1));
        Type t = parse_type(one.substr(colon + 1), line);
        n.shape = t.shape;
        n.dt = t.dt;
        g->params.push_back(add_node(std::move(n), line));
        if (comma == sv::npos) break;
        i = comma + 2;
      }
      continue;
    }
    if (!in_func) perr("statement outside func.func @main", line);
    if (starts(line, "return ")) {
      sv r = line.substr(7);
      size_t colon = r.find(" : ");
      if (colon == sv::npos) perr("bad return", line);
      for (auto& nm : parse_operands(r.substr(0, colon), line)) g->outputs.push_back(lookup(nm, line));
      have_return = true;
      continue;
    }
    if (line[0] != '%') perr("unexpected statement", line);
    size_t eq = line.find(" = ");
    if (eq == sv::npos) perr("expected assignment", line);
    Node n;
    n.name = std::string(line.substr(1, eq - 1));
    sv rhs = line.substr(eq + 3);

    if (starts(rhs, "stablehlo.constant dense<")) {
      size_t tpos = rhs.rfind("> : ");
      if (tpos == sv::npos) perr("bad constant", line);
      Type t = parse_type(rhs.substr(tpos + 4), line);
      n.op = Op::Constant;
      n.shape = t.shape;
      n.dt = t.dt;
      sv lit = rhs.substr(25, tpos - 25);
      const char* c = lit.data();
      const char* e = c + lit.size();
      if (!lit.empty() && lit[0] == '[') {
        std::vector<double> vals;
        c++;
        const char* close = e;
        while (close > c && close[-1] != ']') --close;  // the literal's closing bracket
        if (close > c) --close;
        const size_t len = (size_t)(close - c);
        // large literals (the [S, T] masks and [S, hd] RoPE tables of a
        // static-position prefill) are split at commas over host threads
        const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
        const size_t nthr = len < (1u << 20) ? 1 : std::min<size_t>(hw, std::min<size_t>(32, len >> 18));
        if (nthr <= 1) {
          vals.reserve((size_t)std::max<int64_t>(1, n.numel()));
          parse_values(c, close, vals, line);
        } else {
          std::vector<const char*> cut(nthr + 1);
          cut[0] = c;
          cut[nthr] = close;
          for (size_t t = 1; t < nthr; ++t) {
            const char* q = c + len * t / nthr;
            while (q < close && *q != ',') ++q;
            cut[t] = std::max(q, cut[t - 1]);
          }
          std::vector<std::vector<double>> parts(nthr);
          std::vector<std::string> errs(nthr);
          std::vector<std::thread> th;
          for (size_t t = 0; t < nthr; ++t)
            th.emplace_back([&, t] {
              try {
                parts[t].reserve((size_t)(cut[t + 1] - cut[t]) / 8 + 1);
                parse_values(cut[t], cut[t + 1], parts[t], line);
              } catch (const std::exception& x) {
                errs[t] = x.what();
              }
            });
          for (auto& x : th) x.join();
          for (const auto& m : errs)
            if (!m.empty()) perr("bad literal value", line);
          size_t tot = 0;
          for (const auto& v : parts) tot += v.size();
          vals.reserve(tot);
          for (auto& v : parts) vals.insert(vals.end(), v.begin(), v.end());
        }
        if ((int64_t)vals.size() != n.numel()) perr("dense literal has wrong element count", line);
        store_literal(n, vals);
      } else {
        n.splat = true;
        n.splat_val = round_to_dt(parse_scalar_token(c, e, line), n.dt);
      }
      add_node(std::move(n), line);
      continue;
    }
    if (starts(rhs, "stablehlo.reshape ")) {
      sv r = rhs.substr(18);
      size_t colon = r.find(" : ");
      size_t arrow = r.rfind(" -> ");
      if (colon == sv::npos || arrow == sv::npos) perr("bad reshape", line);
      auto ops = parse_operands(r.substr(0, colon), line);
      Type t = parse_type(r.substr(arrow + 4), line);
      n.op = Op::Reshape;
      n.in = {lookup(ops.at(0), line)};
      n.shape = t.shape;
      n.dt = t.dt;
      if (numel(t.shape) != g->nodes[n.in[0]].numel()) perr("reshape changes element count", line);
      add_node(std::move(n), line);
      continue;
    }
    if (starts(rhs, "\"stablehlo.all_reduce\"(")) {
      // tensor-parallel sum or maximum: region of one stablehlo.add / stablehlo.maximum,
      // replica_groups = dense<[[0, .., n-1]]>
      sv args = rhs.substr(23);
      size_t close = args.find(')');
      auto ops = parse_operands(args.substr(0, close), line);
      if (ops.size() != 1) perr("all_reduce expects 1 operand", line);
      sv body_line, tail_line;
      for (int k = 0; k < 3 && p < end; ++k) {
        const char* nl2 = (const char*)memchr(p, '\n', (size_t)(end - p));
        if (!nl2) nl2 = end;
        sv l2 = trim(sv(p, (size_t)(nl2 - p)));
        p = nl2 + 1;
        if (k == 1) body_line = l2;
        if (k == 2 && !starts(l2, "\"stablehlo.return\"")) perr("unexpected all_reduce region", l2);
      }
      {
        const char* nl2 = (const char*)memchr(p, '\n', (size_t)(end - p));
        if (!nl2) nl2 = end;
        tail_line = trim(sv(p, (size_t)(nl2 - p)));
        p = nl2 + 1;
      }
      int64_t red = RED_ADD;
      if (body_line.find("stablehlo.maximum ") != sv::npos) red = RED_MAX;
      else if (body_line.find("stablehlo.add ") == sv::npos)
        fail(E_UNIMPLEMENTED, "all_reduce body not supported: " + std::string(body_line));
      if (!starts(tail_line, "})")) perr("bad all_reduce tail", tail_line);
      size_t g = tail_line.find("replica_groups = dense<[[");
      if (g == sv::npos) perr("all_reduce without replica_groups", tail_line);
      sv grp = tail_line.substr(g + 25);
      size_t ge = grp.find("]]");
      if (ge == sv::npos) perr("bad replica_groups", tail_line);
      int64_t count = 1;
      for (char c : grp.substr(0, ge)) count += c == ',';
      size_t arrow = tail_line.rfind(" -> ");
      Type t = parse_type(tail_line.substr(arrow + 4), tail_line);
      n.op = Op::AllReduce;
      n.i0 = count;
      n.ia = {red};
      n.in = {lookup(ops[0], line)};
      n.shape = t.shape;
      n.dt = t.dt;
      add_node(std::move(n), line);
      continue;
    }
    if (starts(rhs, "\"stablehlo.reduce\"(")) {
      // region lines: ^bb0(..):, %arg_res = stablehlo.add|maximum .., "stablehlo.return"(..), }) {...} : .. -> T
      sv args = rhs.substr(19);
      size_t close = args.find(')');
      auto ops = parse_operands(args.substr(0, close), line);
      if (ops.size() != 2) perr("reduce expects 2 operands", line);
      sv body_line, tail_line;
      for (int k = 0; k < 3 && p < end; ++k) {
        const char* nl2 = (const char*)memchr(p, '\n', (size_t)(end - p));
        if (!nl2) nl2 = end;
        sv l2 = trim(sv(p, (size_t)(nl2 - p)));
        p = nl2 + 1;
        if (k == 1) body_line = l2;
        if (k == 2 && !starts(l2, "\"stablehlo.return\"")) perr("unexpected reduce region", l2);
      }
      {
        const char* nl2 = (const char*)memchr(p, '\n', (size_t)(end - p));
        if (!nl2) nl2 = end;
        tail_line = trim(sv(p, (size_t)(nl2 - p)));
        p = nl2 + 1;
      }
      if (body_line.find("stablehlo.add ") != sv::npos) n.i0 = RED_ADD;
      else if (body_line.find("stablehlo.maximum ") != sv::npos) n.i0 = RED_MAX;
      else fail(E_UNIMPLEMENTED, "reduce body not supported: " + std::string(body_line));
      if (!starts(tail_line, "})")) perr("bad reduce tail", tail_line);
      n.ia = attr_list(tail_line, "dimensions", tail_line);
      size_t arrow = tail_line.rfind(" -> ");
      Type t = parse_type(tail_line.substr(arrow + 4), tail_line);
      n.op = Op::Reduce;
      n.in = {lookup(ops[0], line), lookup(ops[1], line)};
      n.shape = t.shape;
      n.dt = t.dt;
      add_node(std::move(n), line);
      continue;
    }
    if (starts(rhs, "\"stablehlo.")) {
      size_t q = rhs.find('"', 1);
      std::string opn(rhs.substr(11, q - 11));
      sv rest = rhs.substr(q + 1);
      if (rest.empty() || rest[0] != '(') perr("expected operand list", line);
      size_t close = rest.find(')');
      auto ops = parse_operands(rest.substr(1, close - 1), line);
      rest = trim(rest.substr(close + 1));
      sv attrs;
      if (!rest.empty() && rest[0] == '{') {
        int depth = 0;
        size_t j = 0;
        for (; j < rest.size(); ++j) {
          if (rest[j] == '{') depth++;
          else if (rest[j] == '}') { if (--depth == 0) break; }
        }
        attrs = rest.substr(1, j - 1);
        rest = trim(rest.substr(j + 1));
      }
      size_t arrow = rest.rfind(" -> ");
      if (!starts(rest, ": ") || arrow == sv::npos) perr("expected function type", line);
      Type t = parse_type(rest.substr(arrow + 4), line);
      n.shape = t.shape;
      n.dt = t.dt;
      for (auto& o : ops) n.in.push_back(lookup(o, line));
      if (opn == "convert") {
        n.op = Op::Convert;
      } else if (opn == "compare") {
        n.op = Op::Compare;
        size_t dp = attrs.rfind("comparison_direction ");
        if (dp == sv::npos) perr("compare without direction", line);
        sv d = attrs.substr(dp + 21, 2);
        if (d == "EQ") n.i0 = CMP_EQ;
        else if (d == "NE") n.i0 = CMP_NE;
        else if (d == "GE") n.i0 = CMP_GE;
        else if (d == "GT") n.i0 = CMP_GT;
        else if (d == "LE") n.i0 = CMP_LE;
        else if (d == "LT") n.i0 = CMP_LT;
        else perr("bad comparison direction", line);
      } else if (opn == "select") {
        n.op = Op::Select;
      } else if (opn == "gather") {
        n.op = Op::Gather;
        n.ia = attr_list(attrs, "offset_dims", line);
        n.ib = attr_list(attrs, "collapsed_slice_dims", line);
        n.ic = attr_list(attrs, "start_index_map", line);
        n.i0 = attr_int(attrs, "index_vector_dim", line);
        n.id = attr_list(attrs, "slice_sizes", line);
      } else if (opn == "transpose") {
        n.op = Op::Transpose;
        n.ia = attr_list(attrs, "permutation", line);
      } else if (opn == "broadcast_in_dim") {
        n.op = Op::Broadcast;
        n.ia = attr_list(attrs, "broadcast_dimensions", line);
      } else if (opn == "slice") {
        n.op = Op::Slice;
        n.ia = attr_list(attrs, "start_indices", line);
        n.ib = attr_list(attrs, "limit_indices", line);
        n.ic = attr_list(attrs, "strides", line);
      } else if (opn == "dynamic_update_slice") {
        n.op = Op::DUS;
      } else if (opn == "iota") {
        n.op = Op::Iota;
        n.i0 = attr_int(attrs, "iota_dimension", line);
      } else if (opn == "concatenate") {
        n.op = Op::Concat;
        n.i0 = attr_int(attrs, "dimension", line);
      } else if (opn == "custom_call") {
        // only the debug module's assertions (stablehlo.clj:562-570)
        size_t tp = attrs.find("call_target_name = \"");
        sv target = tp == sv::npos ? sv() : attrs.substr(tp + 20);
        target = target.substr(0, target.find('"'));
        if (target == "check_non_nan") n.i0 = 0;
        else if (target == "check_non_inf") n.i0 = 1;
        else fail(E_UNIMPLEMENTED, "custom_call target not supported: " + std::string(target));
        if (n.in.size() != 1 || n.dt != DT::I1 || !n.shape.empty()) perr("bad check custom_call", line);
        n.op = Op::NanCheck;
      } else if (opn == "dot_general") {
        n.op = Op::Dot;
        n.ia = attr_list(attrs, "lhs_batching_dimensions", line, false);
        n.ib = attr_list(attrs, "rhs_batching_dimensions", line, false);
        n.ic = attr_list(attrs, "lhs_contracting_dimensions", line);
        n.id = attr_list(attrs, "rhs_contracting_dimensions", line);
      } else {
        fail(E_UNIMPLEMENTED, "unsupported op stablehlo." + opn);
      }
      add_node(std::move(n), line);
      continue;
    }
    if (starts(rhs, "stablehlo.")) {
      sv r = rhs.substr(10);
      size_t sp = r.find(' ');
      std::string opn(r.substr(0, sp));
      sv rest = r.substr(sp + 1);
      size_t colon = rest.rfind(" : ");
      if (colon == sv::npos) perr("expected result type", line);
      auto ops = parse_operands(rest.substr(0, colon), line);
      Type t = parse_type(rest.substr(colon + 3), line);
      n.shape = t.shape;
      n.dt = t.dt;
      static const std::pair<const char*, Op> table[] = {
          {"add", Op::Add}, {"subtract", Op::Sub}, {"multiply", Op::Mul}, {"divide", Op::Div},
          {"maximum", Op::Max}, {"minimum", Op::Min}, {"exponential", Op::Exp}, {"tanh", Op::Tanh},
          {"sqrt", Op::Sqrt}, {"rsqrt", Op::Rsqrt}, {"sine", Op::Sin}, {"cosine", Op::Cos},
          {"logistic", Op::Logistic}, {"negate", Op::Neg}, {"abs", Op::Abs}};
      bool found = false;
      for (auto& kv : table)
        if (opn == kv.first) { n.op = kv.second; found = true; break; }
      if (!found) fail(E_UNIMPLEMENTED, "unsupported op stablehlo." + opn);
      for (auto& o : ops) n.in.push_back(lookup(o, line));
      int want = op_is_unary_math(n.op) ? 1 : 2;
      if ((int)n.in.size() != want) perr("wrong operand count for " + opn, line);
      for (int x : n.in)
        if (g->nodes[x].shape != n.shape) perr("elementwise operand shape mismatch", line);
      add_node(std::move(n), line);
      continue;
    }
    perr("unsupported statement", line);
  }
  if (!have_return) fail(E_INVALID, "MLIR parse error: module has no return");
  return g;
}

}  // namespace cljxla
