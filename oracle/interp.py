"""CPU oracle: a numpy interpreter of the StableHLO text printed by clj-xla.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the B200 library; it
is imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` and never by the product path.

What it restates: the execution semantics the reference obtains from its CPU
PJRT plugin (``xla_cpu_pjrt`` 0.0.1, scripts/fetch_pjrt_binaries.clj:12-15 - a
third-party binary that is not vendored) for the op set printed by
``src/clj_xla/stablehlo.clj:248-600``.  StableHLO op definitions, applied as:

* every floating op computes in f32 (sums in f64) and rounds its result to the
  declared element type (round-to-nearest-even), modelling XLA-CPU's bf16
  float normalisation;
* ``reduce`` folds the printed init value (0 or -1e30, stablehlo.clj:450-452)
  into the result;
* ``gather`` start indices and ``dynamic_update_slice`` start indices are
  clamped so the slice stays in bounds (StableHLO spec);
* ``dot_general`` of mixed operand types (f32 x bf16, as printed for the
  attention context product) promotes both operands to f32; the result takes
  the printed result type.

Parity pin: the printed text this interpreter executes is pinned to the
reference's own examples (README.md:50-55 graph, pjrt_test.clj:37-41,
compile_test.clj:12-16, rocm_e2e_test.clj:38-51) and the one numeric
known-answer test in the reference (rocm_e2e_test.clj:38-51, ``y = 2.5 x``,
x = 0..15) - see tests/test_oracle.py.  No reference test pins model outputs
(the reference's own model tests check traced shapes only).  At model level the
interpreter is pinned to the Hugging Face ``transformers`` implementations of
GPT-2, Gemma-2 and Gemma-3, the anchor of the reference's verification scripts
(verification/verify_torch_vs_clojure.py): f32 logits of a prefill and cached
decode steps agree within 1e-4 on the same weights (tests/test_oracle_hf.py).
"""
from __future__ import annotations

import re
from typing import Dict, List, Tuple

import numpy as np

# ---------------------------------------------------------------- dtypes
_FLOAT = {"f32", "bf16", "f16", "f64"}
_INT = {"i32": np.int32, "i64": np.int64, "i8": np.int8, "i16": np.int16, "ui8": np.uint8,
        "u8": np.uint8, "u32": np.uint32}


def round_bf16(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bfloat16 value, kept in a float32 array."""
    a = np.asarray(a, dtype=np.float32, order="C")
    u = a.view(np.uint32)
    r = (u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) & np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    if np.isnan(a).any():
        out = np.where(np.isnan(a), np.float32(np.nan), out)
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    return (round_bf16(a).view(np.uint32) >> 16).astype(np.uint16)


def to_dtype(a, dt: str) -> np.ndarray:
    """Round / convert an array to the value set of element type ``dt``."""
    if dt == "f32":
        return np.asarray(a, dtype=np.float32)
    if dt == "bf16":
        return round_bf16(np.asarray(a, dtype=np.float32))
    if dt == "f16":
        return np.asarray(a, dtype=np.float16)
    if dt == "f64":
        return np.asarray(a, dtype=np.float64)
    if dt == "i1":
        return np.asarray(a).astype(bool)
    if dt in _INT:
        a = np.asarray(a)
        if a.dtype.kind == "f":
            a = np.trunc(a)
        return a.astype(_INT[dt])
    raise ValueError(f"unsupported element type {dt}")


def np_compute(a: np.ndarray) -> np.ndarray:
    """Operand in its compute precision (floats widen to f32)."""
    if a.dtype in (np.float16,):
        return a.astype(np.float32)
    return a


# ----------------------------------------------------------------- types
_TYPE_RE = re.compile(r"tensor<([0-9x]*?)x?([a-z]+[0-9]*)>")


def parse_type(s: str) -> Tuple[Tuple[int, ...], str]:
    s = s.strip()
    m = re.fullmatch(r"tensor<(?:((?:\d+x)+))?([a-z]+[0-9]*)>", s)
    if not m:
        raise ValueError(f"bad type {s!r}")
    dims = tuple(int(d) for d in m.group(1).split("x") if d) if m.group(1) else ()
    return dims, m.group(2)


def _split_top(s: str) -> List[str]:
    """Split on commas not nested in <> () [] {}."""
    out, depth, cur = [], 0, []
    for ch in s:
        if ch in "<([{":
            depth += 1
        elif ch in ">)]}":
            depth -= 1
        if ch == "," and depth == 0:
            out.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if cur:
        out.append("".join(cur))
    return [x.strip() for x in out if x.strip()]


def _ints(s: str) -> List[int]:
    return [int(x) for x in re.findall(r"-?\d+", s)]


class Op:
    __slots__ = ("name", "out", "args", "attrs", "types", "rtype", "body")

    def __init__(self, name, out, args, attrs, types, rtype, body=None):
        self.name, self.out, self.args, self.attrs = name, out, args, attrs
        self.types, self.rtype, self.body = types, rtype, body


class Module:
    def __init__(self, name, params, ret_types, ops, returns):
        self.name, self.params, self.ret_types, self.ops, self.returns = name, params, ret_types, ops, returns


_LOC = re.compile(r'\s+loc\("[^"]*"\)\s*$')


def parse_module(text: str) -> Module:
    lines = text.split("\n")
    i = 0
    name = None
    params: List[Tuple[str, Tuple]] = []
    ret_types = []
    ops: List[Op] = []
    returns: List[str] = []
    while i < len(lines):
        ln = _LOC.sub("", lines[i].rstrip())
        s = ln.strip()
        i += 1
        if not s or s == "}":
            continue
        if s.startswith("module @"):
            name = s[len("module @"):].split()[0]
            continue
        if s.startswith("func.func @main("):
            sig = s[len("func.func @main("):]
            depth, j = 1, 0
            while depth:
                if sig[j] == "(":
                    depth += 1
                elif sig[j] == ")":
                    depth -= 1
                j += 1
            for p in _split_top(sig[:j - 1]):
                pn, pt = p.split(":", 1)
                params.append((pn.strip()[1:], parse_type(pt)))
            rest = sig[j:].strip()
            m = re.match(r"->\s*\((.*)\)\s*\{$", rest)
            ret_types = [parse_type(x) for x in _split_top(m.group(1))]
            continue
        if s.startswith("return "):
            body = s[len("return "):]
            names, _ = body.split(" : ", 1)
            returns = [x.strip()[1:] for x in names.split(",")]
            continue
        m = re.match(r"%([\w.]+) = (.*)$", s)
        if not m:
            raise ValueError(f"cannot parse line: {s!r}")
        out, rhs = m.group(1), m.group(2)
        if rhs.startswith('"stablehlo.reduce"('):
            # region: ^bb0 line, body op line, return line, closing line with attrs/type
            body_line = lines[i + 1].strip()
            close = lines[i + 3].strip()
            i += 4
            body_op = re.match(r"%arg_res = (stablehlo\.\w+)", body_line).group(1)
            args = re.findall(r"%([\w.]+)", rhs[len('"stablehlo.reduce"('):].split(")")[0])
            dims = _ints(re.search(r"dimensions = array<i64:([^>]*)>", close).group(1))
            sig = close.split("} : ", 1)[1]
            ins, rt = sig.split(" -> ")
            ops.append(Op("reduce", out, args, {"dimensions": dims}, None, parse_type(rt), body_op))
            continue
        if rhs.startswith('"stablehlo.all_reduce"('):
            body_line = lines[i + 1].strip()
            close = lines[i + 3].strip()
            i += 4
            body_op = re.match(r"%arg_res = (stablehlo\.\w+)", body_line).group(1)
            args = re.findall(r"%([\w.]+)", rhs[len('"stablehlo.all_reduce"('):].split(")")[0])
            groups = re.search(r"replica_groups = dense<\[\[([^\]]*)\]\]>", close).group(1)
            rt = close.rsplit(" -> ", 1)[1]
            ops.append(Op("all_reduce", out, args, {"replicas": len(_ints(groups))}, None, parse_type(rt), body_op))
            continue
        if rhs.startswith("stablehlo.constant dense<"):
            lit, rt = rhs[len("stablehlo.constant dense<"):].rsplit("> : ", 1)
            ops.append(Op("constant", out, [], {"literal": lit}, None, parse_type(rt)))
            continue
        if rhs.startswith("stablehlo.reshape "):
            a, sig = rhs[len("stablehlo.reshape "):].split(" : ", 1)
            rt = sig.split(" -> ")[1]
            ops.append(Op("reshape", out, [a.strip()[1:]], {}, None, parse_type(rt)))
            continue
        if rhs.startswith('"stablehlo.'):
            opname = rhs[len('"stablehlo.'):rhs.index('"', 1)]
            rest = rhs[rhs.index('"', 1) + 1:]
            assert rest.startswith("(")
            close = rest.index(")")
            args = [x.strip()[1:] for x in rest[1:close].split(",") if x.strip()]
            rest = rest[close + 1:].strip()
            attrs = {}
            if rest.startswith("{"):
                depth, j = 0, 0
                while True:
                    if rest[j] == "{":
                        depth += 1
                    elif rest[j] == "}":
                        depth -= 1
                        if depth == 0:
                            break
                    j += 1
                attrs = {"raw": rest[1:j]}
                rest = rest[j + 1:].strip()
            assert rest.startswith(": "), rest
            rt = rest.rsplit(" -> ", 1)[1]
            ops.append(Op(opname, out, args, attrs, None, parse_type(rt)))
            continue
        if rhs.startswith("stablehlo."):
            opname = rhs[len("stablehlo."):].split()[0]
            body = rhs[len("stablehlo.") + len(opname):]
            argstr, rt = body.rsplit(" : ", 1)
            args = [x.strip()[1:] for x in argstr.split(",") if x.strip()]
            ops.append(Op(opname, out, args, {}, None, parse_type(rt)))
            continue
        raise ValueError(f"unsupported op line: {s!r}")
    return Module(name, params, ret_types, ops, returns)


# ------------------------------------------------------------- execution
def _parse_literal(lit: str, shape, dt) -> np.ndarray:
    lit = lit.strip()
    n = int(np.prod(shape)) if shape else 1
    if lit.startswith("["):
        body = lit[1:-1].strip()
        if dt in _FLOAT:
            vals = np.array([float(x) for x in body.split(",")] if body else [], dtype=np.float64)
        else:
            vals = np.array([int(x) for x in body.split(",")] if body else [], dtype=np.int64)
        if vals.size != n:
            raise ValueError("dense literal size mismatch")
        arr = vals.reshape(shape)
    else:
        # a splat: convert the one value, then a read-only broadcast view (every
        # op makes a new array for its result, so the view is never written)
        v = float(lit) if dt in _FLOAT else int(lit)
        one = np.array(v, dtype=np.float64 if dt in _FLOAT else np.int64)
        if dt in _FLOAT:
            one = _f64_to_bf16(one) if dt == "bf16" else to_dtype(one, dt)
        else:
            one = to_dtype(one, dt)
        return np.broadcast_to(one, shape)
    if dt in _FLOAT:
        # decimal -> nearest f64 -> nearest value of the element type
        if dt == "bf16":
            return _f64_to_bf16(arr)
        return to_dtype(arr, dt)
    return to_dtype(arr, dt)


def _f64_to_bf16(a: np.ndarray) -> np.ndarray:
    """Correctly rounded f64 -> bf16 (avoids f64->f32->bf16 double rounding)."""
    a = np.asarray(a, dtype=np.float64)
    f = a.astype(np.float32)
    lo = np.atleast_1d(round_bf16(f))   # arrays: unsigned wrap-around below is silent and masked
    # candidate neighbours in bf16 spacing around the f32 rounding; the one below
    # a zero is the smallest bf16 of the opposite sign
    u = lo.view(np.uint32)
    up = (u + np.uint32(0x10000)).view(np.float32)
    at_zero = (u & np.uint32(0x7FFFFFFF)) == 0
    dn = np.where(at_zero, (u ^ np.uint32(0x80000000)) | np.uint32(0x10000),
                  u - np.uint32(0x10000)).astype(np.uint32).view(np.float32)
    a = a.reshape(lo.shape)
    best = lo.copy()
    err = np.abs(a - lo.astype(np.float64))
    for c in (up, dn):
        e = np.abs(a - c.astype(np.float64))
        better = e < err
        tie = (e == err) & ((c.view(np.uint32) >> 16) & 1 == 0)
        sel = better | tie
        best = np.where(sel, c, best)
        err = np.where(sel, e, err)
    return best.astype(np.float32).reshape(f.shape)


def _ew(fn, args, rdt):
    xs = [np_compute(a) for a in args]
    if rdt in _FLOAT:
        xs = [x.astype(np.float32) for x in xs]
        with np.errstate(all="ignore"):
            return to_dtype(fn(*xs), rdt)
    with np.errstate(all="ignore"):
        return to_dtype(fn(*xs), rdt)


def _int_div(a, b):
    q = np.trunc(np.divide(a.astype(np.float64), b.astype(np.float64)))
    return q


class Interpreter:
    """Executes a parsed module; ``run`` returns the outputs (and optionally every SSA value).

    ``ulp_noise_seed``: when set, the f32 accumulation of every ``dot_general``
    and sum-reduce is moved by a seeded random number of f32 ulps before it is
    rounded to the result type - a model of a different, equally valid f32
    summation order - and every exp / tanh / sin / cos result by up to 2 ulps
    (a different, equally valid math library: the CUDA math library documents
    2-ulp bounds for these functions).  Two orders of an n-term f32 sum differ by about
    sqrt(n)/5 ulps of the result (median over random bf16 products; the 90th
    percentile is 4-6x that), so the shift is normal with that standard
    deviation (at least one ulp).  Tests use the spread it causes as the noise
    floor of a whole bf16 model (see tests/parity.py).
    """

    def __init__(self, text: str, ulp_noise_seed=None, collective=None):
        self.module = parse_module(text) if isinstance(text, str) else text
        self._consts: Dict[str, np.ndarray] = {}
        self._noise = None if ulp_noise_seed is None else np.random.default_rng(ulp_noise_seed)
        # all_reduce: collective(value) -> the sum over the group (see run_mlir_tp)
        self._collective = collective

    def run(self, inputs: List[np.ndarray], keep_all: bool = False):
        m = self.module
        env: Dict[str, np.ndarray] = {}
        if len(inputs) != len(m.params):
            raise ValueError(f"expected {len(m.params)} inputs, got {len(inputs)}")
        for (pn, (shape, dt)), val in zip(m.params, inputs):
            a = np.asarray(val)
            if dt == "bf16" and a.dtype == np.uint16:
                a = bf16_bits_to_f32(a)
            elif not (dt == "bf16" and a.dtype == np.float32):   # f32 arrays of bf16 values pass as-is
                a = to_dtype(a, dt)
            if tuple(a.shape) != tuple(shape):
                a = a.reshape(shape)
            env[pn] = a
        uses: Dict[str, int] = {}
        if not keep_all:
            for op in m.ops:
                for a in op.args:
                    uses[a] = uses.get(a, 0) + 1
            for r in m.returns:
                uses[r] = uses.get(r, 0) + (1 << 30)   # outputs are never freed
        for op in m.ops:
            env[op.out] = self._exec(op, env)
            if not keep_all:
                for a in op.args:
                    uses[a] -= 1
                    if uses[a] == 0 and a not in m.returns:
                        env.pop(a, None)
        outs = [env[r] for r in m.returns]
        return (outs, env) if keep_all else outs

    def _exec(self, op: Op, env):
        shape, dt = op.rtype
        name = op.name
        args = [env[a] for a in op.args]
        if name == "constant":
            c = self._consts.get(op.out)
            if c is None:
                c = _parse_literal(op.attrs["literal"], shape, dt)
                self._consts[op.out] = c
            return c
        if name == "reshape":
            return args[0].reshape(shape)
        if name in ("add", "subtract", "multiply", "divide", "maximum"):
            if dt in _FLOAT:
                fn = {"add": np.add, "subtract": np.subtract, "multiply": np.multiply,
                      "divide": np.divide, "maximum": np.maximum}[name]
            else:
                fn = {"add": np.add, "subtract": np.subtract, "multiply": np.multiply,
                      "divide": _int_div, "maximum": np.maximum}[name]
            return _ew(fn, args, dt)
        if name in ("exponential", "tanh", "sqrt", "sine", "cosine", "logistic", "negate", "abs", "rsqrt"):
            fn = {"exponential": np.exp, "tanh": np.tanh, "sqrt": np.sqrt, "sine": np.sin, "cosine": np.cos,
                  "logistic": lambda x: np.float32(1) / (np.float32(1) + np.exp(-x)),
                  "negate": np.negative, "abs": np.abs,
                  "rsqrt": lambda x: np.float32(1) / np.sqrt(x)}[name]
            if self._noise is not None and dt in _FLOAT and name in ("exponential", "tanh", "sine", "cosine"):
                # a valid f32 library result within its documented error bound
                # (2 ulps for these functions in the CUDA math library)
                x = np.asarray(args[0], np.float32)
                with np.errstate(all="ignore"):
                    r = np.asarray(fn(x), np.float32)
                u = self._noise.integers(-2, 3, size=r.shape)
                r = (r.astype(np.float64) + u * np.spacing(np.abs(r)).astype(np.float64)).astype(np.float32)
                return to_dtype(r, dt)
            return _ew(fn, args, dt)
        if name == "convert":
            a = args[0]
            if dt in _FLOAT:
                if a.dtype.kind in "biu":      # exact integer -> nearest float of the type
                    a64 = a.astype(np.float64)
                    return _f64_to_bf16(a64) if dt == "bf16" else to_dtype(a64, dt)
                return to_dtype(a.astype(np.float32), dt)
            if dt == "i1":
                return a != 0
            if a.dtype.kind == "f":            # float -> int truncates toward zero
                with np.errstate(all="ignore"):
                    return np.trunc(a.astype(np.float64)).astype(_INT[dt])
            return a.astype(_INT[dt])
        if name == "compare":
            d = re.search(r"comparison_direction (\w+)", op.attrs["raw"]).group(1)
            a, b = args
            f = {"EQ": np.equal, "NE": np.not_equal, "GE": np.greater_equal, "GT": np.greater,
                 "LE": np.less_equal, "LT": np.less}[d]
            return f(a, b)
        if name == "select":
            p, a, b = args
            return to_dtype(np.where(p, a, b), dt)
        if name == "broadcast_in_dim":
            bd = _ints(re.search(r"broadcast_dimensions = array<i64:?([^>]*)>", op.attrs["raw"]).group(1))
            a = args[0]
            order = np.argsort(bd)
            a = np.transpose(a, order) if a.ndim else a
            sb = sorted(bd)
            sh = [1] * len(shape)
            for k, dd in enumerate(sb):
                sh[dd] = a.shape[k]
            return np.broadcast_to(a.reshape(sh), shape)
        if name == "transpose":
            perm = _ints(re.search(r"permutation = array<i64:([^>]*)>", op.attrs["raw"]).group(1))
            return np.transpose(args[0], perm)
        if name == "slice":
            raw = op.attrs["raw"]
            lim = _ints(re.search(r"limit_indices = array<i64:([^>]*)>", raw).group(1))
            st = _ints(re.search(r"start_indices = array<i64:([^>]*)>", raw).group(1))
            sd = _ints(re.search(r"strides = array<i64:([^>]*)>", raw).group(1))
            return args[0][tuple(slice(s, l, k) for s, l, k in zip(st, lim, sd))]
        if name == "concatenate":
            dim = int(re.search(r"dimension = (-?\d+)", op.attrs["raw"]).group(1))
            return to_dtype(np.concatenate(args, axis=dim), dt)
        if name == "iota":
            idim = int(re.search(r"iota_dimension = (\d+)", op.attrs["raw"]).group(1))
            r = np.arange(shape[idim])
            sh = [1] * len(shape)
            sh[idim] = shape[idim]
            return to_dtype(np.broadcast_to(r.reshape(sh), shape), dt)
        if name == "dynamic_update_slice":
            base, upd = args[0], args[1]
            starts = [int(np.asarray(s).reshape(())) for s in args[2:]]
            out = np.array(base, copy=True)
            idx = []
            for d, s in enumerate(starts):
                s = min(max(s, 0), base.shape[d] - upd.shape[d])
                idx.append(slice(s, s + upd.shape[d]))
            out[tuple(idx)] = upd
            return out
        if name == "custom_call":
            # the debug module's assertions (debug.clj:24-60, printed at
            # stablehlo.clj:562-570): true when no element is NaN / infinite
            raw = op.attrs.get("raw", "")
            x = np.asarray(args[0], np.float64)
            if 'call_target_name = "check_non_nan"' in raw:
                return np.array(not np.isnan(x).any())
            if 'call_target_name = "check_non_inf"' in raw:
                return np.array(not np.isinf(x).any())
            raise NotImplementedError(f"oracle: custom_call {raw}")
        if name == "all_reduce":
            if self._collective is None:
                raise ValueError("all_reduce needs the ranks of its group (run_mlir_tp)")
            kind = "max" if op.body == "stablehlo.maximum" else "sum"
            x = np.asarray(args[0], np.int64 if dt in _INT else np.float32)
            return to_dtype(self._collective(x, kind), dt)
        if name == "gather":
            return self._gather(op, args, shape, dt)
        if name == "reduce":
            r = self._reduce(op, args, shape, dt)
            return r
        if name == "dot_general":
            return self._dot(op, args, shape, dt)
        raise NotImplementedError(f"oracle: op {name} not supported")

    def _ulp_noise(self, r, n_terms=1):
        """Summation-order noise on an f32 accumulation of n_terms terms, before its
        rounding to the result type: a normal number of ulps, sigma max(1, sqrt(n)/5)."""
        if self._noise is None:
            return r
        r = np.asarray(r, np.float32)
        sigma = max(1.0, float(np.sqrt(max(1, n_terms))) / 5.0)
        u = np.rint(self._noise.normal(0.0, sigma, size=r.shape))
        return (r.astype(np.float64) + u * np.spacing(np.abs(r)).astype(np.float64)).astype(np.float32)

    def _gather(self, op, args, shape, dt):
        raw = op.attrs["raw"]
        offset = _ints(re.search(r"offset_dims = \[([^\]]*)\]", raw).group(1))
        collapsed = _ints(re.search(r"collapsed_slice_dims = \[([^\]]*)\]", raw).group(1))
        smap = _ints(re.search(r"start_index_map = \[([^\]]*)\]", raw).group(1))
        ivd = int(re.search(r"index_vector_dim = (\d+)", raw).group(1))
        sizes = _ints(re.search(r"slice_sizes = array<i64:([^>]*)>", raw).group(1))
        operand, idx = args
        if not (collapsed == [0] and smap == [0] and operand.ndim == 2 and sizes[0] == 1
                and sizes[1] == operand.shape[1] and ivd == idx.ndim - 1 and idx.shape[-1] == 1
                and offset == [idx.ndim - 1]):
            raise NotImplementedError("oracle: gather form not supported")
        rows = np.clip(idx[..., 0].astype(np.int64), 0, operand.shape[0] - 1)
        return operand[rows].reshape(shape)

    def _reduce(self, op, args, shape, dt):
        a, init = args
        dims = tuple(op.attrs["dimensions"])
        if op.body == "stablehlo.add":
            if dt in _FLOAT:
                r = np.sum(a.astype(np.float64), axis=dims) + float(init)
            else:
                r = np.sum(a.astype(np.int64), axis=dims) + int(init)
        else:
            if dt in _FLOAT:
                r = np.maximum(np.max(a, axis=dims).astype(np.float64), float(init))
            else:
                r = np.maximum(np.max(a, axis=dims), init)
        r = np.asarray(r).reshape(shape)
        if op.body == "stablehlo.add" and dt in _FLOAT and self._noise is not None:
            r = self._ulp_noise(r.astype(np.float32), int(np.prod([a.shape[d] for d in dims])) if dims else 1)
        return to_dtype(r, dt)

    def _dot(self, op, args, shape, dt):
        raw = op.attrs["raw"]

        def grab(key):
            m = re.search(key + r" = \[([^\]]*)\]", raw)
            return _ints(m.group(1)) if m else []

        lb, rb = grab("lhs_batching_dimensions"), grab("rhs_batching_dimensions")
        lc, rc = grab("lhs_contracting_dimensions"), grab("rhs_contracting_dimensions")
        a, b = args
        lf = [i for i in range(a.ndim) if i not in lb and i not in lc]
        rf = [i for i in range(b.ndim) if i not in rb and i not in rc]
        if not lb and not rb and b.ndim == 2 and len(lc) == 1 and lc[0] == a.ndim - 1:
            # plain linear layer: a[..., K] x b (a 2-D view, possibly transposed) - no copies
            bt = np.asarray(b, np.float32)
            bt = bt if rc[0] == 0 else bt.T
            r = np.asarray(a, np.float32).reshape(-1, a.shape[-1]) @ bt
            return to_dtype(self._ulp_noise(r.reshape(shape), a.shape[-1]), dt)
        at = np.asarray(np.transpose(a, lb + lf + lc), np.float32)
        bt = np.asarray(np.transpose(b, rb + rc + rf), np.float32)
        bsz = int(np.prod([a.shape[i] for i in lb])) if lb else 1
        m = int(np.prod([a.shape[i] for i in lf])) if lf else 1
        k = int(np.prod([a.shape[i] for i in lc])) if lc else 1
        n = int(np.prod([b.shape[i] for i in rf])) if rf else 1
        r = np.matmul(at.reshape(bsz, m, k), bt.reshape(bsz, k, n))
        return to_dtype(self._ulp_noise(r.reshape(shape), k), dt)


def run_mlir(text: str, inputs, keep_all=False, ulp_noise_seed=None):
    return Interpreter(text, ulp_noise_seed).run(inputs, keep_all=keep_all)


def run_mlir_tp(texts, inputs_per_rank, ulp_noise_seed=None):
    """Runs the per-rank graphs of a tensor-parallel group together, one thread
    per rank.  Each all_reduce is the sum, in f64 and in rank order, of the
    ranks' f32 values, rounded to the result type by the caller's op, or (a
    ``stablehlo.maximum`` region) their elementwise maximum."""
    import threading
    n = len(texts)
    barrier = threading.Barrier(n)
    slots = [None] * n
    result = [None]
    outs = [None] * n
    errors = []

    def worker(r):
        def collective(x, kind="sum"):
            slots[r] = x
            barrier.wait()
            if r == 0:
                if kind == "max":
                    result[0] = np.maximum.reduce([np.asarray(v) for v in slots])
                else:
                    acc = np.zeros(x.shape, np.float64)
                    for v in slots:
                        acc += v
                    result[0] = acc
            barrier.wait()
            y = result[0]
            barrier.wait()
            return y
        try:
            seed = None if ulp_noise_seed is None else ulp_noise_seed + 1000 * r
            outs[r] = Interpreter(texts[r], seed, collective).run(inputs_per_rank[r])
        except Exception as e:  # noqa: BLE001 - reported after the join
            errors.append(e)
            barrier.abort()

    threads = [threading.Thread(target=worker, args=(r,)) for r in range(n)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    if errors:
        raise errors[0]
    return outs
