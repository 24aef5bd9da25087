"""Symbolic tracer: records tensor operations as EDN-style SSA equations.

This is the host-side mirror of clj-xla's tracing DSL for the decoder path:
``src/clj_xla/tensor.clj`` (Tracer record, scalar auto-lifting, numpy-style
broadcasting through explicit ``broadcast_in_dim``, every op constructor) and
``src/clj_xla/trace.clj:6-22`` (``trace-graph``).

The equations it records are consumed by :mod:`stablehlo` (the MLIR printer),
whose text is the contract handed to the B200 library.  Everything here keeps
the reference's observable behaviour: variable naming (``prefix_<counter>``),
equation order, the *tracer-side* types (which may differ from the printer's
re-inferred types - the reference has the same split) and the attribute maps.

Types are ``("tensor", shape_tuple, dtype_str)``; dtype strings are the
reference keywords without the colon (``"f32"``, ``"bf16"``, ``"i32"``, ``"i1"``).
"""
from __future__ import annotations

import math
from typing import Any, List, Optional, Sequence


class Tracer:
    """A symbolic SSA value (tensor.clj:5 ``defrecord Tracer [id type]``)."""

    __slots__ = ("id", "type")

    def __init__(self, id: str, type: tuple):
        self.id = id
        self.type = (type[0], tuple(type[1]), type[2])

    @property
    def shape(self):
        return self.type[1]

    @property
    def dtype(self):
        return self.type[2]

    def __repr__(self):
        return f"Tracer({self.id!r}, {self.type!r})"


class _TraceCtx:
    def __init__(self):
        self.eqns: List[dict] = []
        self.counter = 0


_CTX: Optional[_TraceCtx] = None
_GENSYM = [1000]


def tracer_p(v) -> bool:
    return isinstance(v, Tracer)


def _is_number(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def gen_var_id(prefix: str) -> str:
    """tensor.clj:14-17 - ``prefix_<n>`` with a per-trace counter starting at 1."""
    if _CTX is not None:
        _CTX.counter += 1
        return f"{prefix}_{_CTX.counter}"
    _GENSYM[0] += 1
    return f"{prefix}_G__{_GENSYM[0]}"


def _emit(eqn: dict):
    if _CTX is not None:
        _CTX.eqns.append(eqn)


def emit_constant(val, target_type=None) -> Tracer:
    """tensor.clj:19-43 - lift a number / nested vector into a constant equation."""
    if tracer_p(val):
        return val
    if _is_number(val):
        out_id = gen_var_id("c")
        out_type = target_type or ("tensor", (), "f32")
        _emit({"op": "stablehlo/constant", "outvars": [out_id], "value": val, "type": out_type})
        return Tracer(out_id, out_type)
    if isinstance(val, (list, tuple)):
        out_id = gen_var_id("c_vec")
        out_type = target_type or ("tensor", (128, 128), "f32")
        _emit({"op": "stablehlo/constant", "outvars": [out_id], "value": val, "type": out_type})
        return Tracer(out_id, out_type)
    raise ValueError(f"Cannot emit constant for unsupported value {val!r}")


def _broadcast_shapes(a: Sequence[int], b: Sequence[int]) -> tuple:
    """tensor.clj:47-53 - left-pad with ones, elementwise max."""
    r = max(len(a), len(b))
    pa = (1,) * (r - len(a)) + tuple(a)
    pb = (1,) * (r - len(b)) + tuple(b)
    return tuple(max(x, y) for x, y in zip(pa, pb))


def _binary(op: str, prefix: str, a, b, attrs=None, out_dtype_override=None) -> Tracer:
    """tensor.clj:55-80 ``binary-elementwise-op``.

    A scalar on the right inherits the left operand's full type; a scalar on
    the left is an f32 scalar that gets broadcast (and sets the tracer dtype).
    """
    ta = emit_constant(a, None)
    tb = emit_constant(b, ta.type)
    t_kw, shape_a, dtype_a = ta.type
    shape_b = tb.type[1]
    out_shape = _broadcast_shapes(shape_a, shape_b)
    rank_out = len(out_shape)
    if shape_a == out_shape:
        ta_b = ta
    else:
        ta_b = broadcast_in_dim(ta, out_shape, list(range(rank_out - len(shape_a), rank_out)))
    if shape_b == out_shape:
        tb_b = tb
    else:
        tb_b = broadcast_in_dim(tb, out_shape, list(range(rank_out - len(shape_b), rank_out)))
    out_type = (t_kw, out_shape, out_dtype_override or dtype_a)
    out_id = gen_var_id(prefix)
    eqn = {"op": op, "invars": [ta_b.id, tb_b.id], "outvars": [out_id]}
    if attrs:
        eqn["attrs"] = attrs
    _emit(eqn)
    return Tracer(out_id, out_type)


def add(a, b, *more):
    r = _binary("stablehlo/add", "t_add", a, b)
    for m in more:
        r = add(r, m)
    return r


def sub(a, b=None, *more):
    if b is None:  # unary negation: (- 0.0 a)
        return _binary("stablehlo/subtract", "t_sub", 0.0, a)
    r = _binary("stablehlo/subtract", "t_sub", a, b)
    for m in more:
        r = sub(r, m)
    return r


def mul(a, b, *more):
    r = _binary("stablehlo/multiply", "t_mul", a, b)
    for m in more:
        r = mul(r, m)
    return r


def div(a, b, *more):
    r = _binary("stablehlo/divide", "t_div", a, b)
    for m in more:
        r = div(r, m)
    return r


def _unary(op: str, prefix: str, x) -> Tracer:
    tx = emit_constant(x, None)
    out_id = gen_var_id(prefix)
    _emit({"op": op, "invars": [tx.id], "outvars": [out_id]})
    return Tracer(out_id, tx.type)


def exp(x):
    return _unary("stablehlo/exp", "t_exp", x)


def sqrt(x):
    return _unary("stablehlo/sqrt", "t_sqrt", x)


def rsqrt(x):
    return div(1.0, sqrt(x))


def pow(x, p):
    """tensor.clj:137-148 - p = 2.0 / 3.0 become multiplies."""
    if isinstance(p, float) and p == 2.0:
        return mul(x, x)
    if isinstance(p, float) and p == 3.0:
        return mul(x, mul(x, x))
    tx = emit_constant(x, None)
    out_id = gen_var_id("t_pow")
    _emit({"op": "stablehlo/power", "invars": [tx.id], "outvars": [out_id], "value": p})
    return Tracer(out_id, tx.type)


def maximum(x, y):
    return _binary("stablehlo/maximum", "t_max", x, y)


def tanh(x):
    return _unary("stablehlo/tanh", "t_tanh", x)


def sigmoid(x):
    return _unary("stablehlo/logistic", "t_logistic", x)


def sin(x):
    return _unary("stablehlo/sine", "t_sin", x)


def cos(x):
    return _unary("stablehlo/cosine", "t_cos", x)


def convert(x, target_dtype: str):
    tx = emit_constant(x, None)
    t_kw, shape, _ = tx.type
    out_id = gen_var_id("t_convert")
    _emit({"op": "stablehlo/convert", "invars": [tx.id], "outvars": [out_id],
           "attrs": {"target_dtype": target_dtype}})
    return Tracer(out_id, (t_kw, shape, target_dtype))


def concatenate(tensors, dimension: int):
    tracers = [emit_constant(t, None) for t in tensors]
    t_kw, first_shape, dtype = tracers[0].type
    rank = len(first_shape)
    dim = rank + dimension if dimension < 0 else dimension
    total = sum(t.type[1][dim] for t in tracers)
    out_shape = list(first_shape)
    out_shape[dim] = total
    out_id = gen_var_id("t_concat")
    _emit({"op": "stablehlo/concatenate", "invars": [t.id for t in tracers], "outvars": [out_id],
           "attrs": {"dimension": dim}})
    return Tracer(out_id, (t_kw, tuple(out_shape), dtype))


def dot_general(lhs, rhs, attrs: dict):
    """tensor.clj:229-252; output dtype is the lhs dtype."""
    tl = emit_constant(lhs, None)
    tr = emit_constant(rhs, None)
    t_kw, lshape, dtype = tl.type
    rshape = tr.type[1]
    cd = attrs.get("contracting_dims", {})
    bd = attrs.get("batch_dims", {})
    c_l = set(cd.get("lhs", [len(lshape) - 1]))
    c_r = set(cd.get("rhs", [0]))
    b_l = set(bd.get("lhs", []))
    b_r = set(bd.get("rhs", []))
    batch = [lshape[i] for i in bd.get("lhs", [])]
    lfree = [d for i, d in enumerate(lshape) if i not in c_l and i not in b_l]
    rfree = [d for i, d in enumerate(rshape) if i not in c_r and i not in b_r]
    out_shape = tuple(batch + lfree + rfree)
    out_id = gen_var_id("t_dot")
    _emit({"op": "stablehlo/dot_general", "invars": [tl.id, tr.id], "outvars": [out_id], "attrs": attrs})
    return Tracer(out_id, (t_kw, out_shape, dtype))


def matmul(lhs, rhs):
    tl = emit_constant(lhs, None)
    tr = emit_constant(rhs, None)
    rank = len(tl.type[1])
    return dot_general(tl, tr, {"contracting_dims": {"lhs": [rank - 1], "rhs": [0]}})


def reshape(x, new_shape):
    tx = emit_constant(x, None)
    t_kw, _, dtype = tx.type
    out_type = (t_kw, tuple(new_shape), dtype)
    out_id = gen_var_id("t_reshape")
    _emit({"op": "stablehlo/reshape", "invars": [tx.id], "outvars": [out_id], "type": out_type,
           "attrs": {"shape": list(new_shape)}})
    return Tracer(out_id, out_type)


def transpose(x, permutation):
    tx = emit_constant(x, None)
    t_kw, in_shape, dtype = tx.type
    out_type = (t_kw, tuple(in_shape[p] for p in permutation), dtype)
    out_id = gen_var_id("t_transpose")
    _emit({"op": "stablehlo/transpose", "invars": [tx.id], "outvars": [out_id], "type": out_type,
           "attrs": {"permutation": list(permutation)}})
    return Tracer(out_id, out_type)


def broadcast_in_dim(x, target_shape, bcast_dims):
    tx = emit_constant(x, None)
    t_kw, _, dtype = tx.type
    out_id = gen_var_id("t_bcast")
    out_type = (t_kw, tuple(target_shape), dtype)
    _emit({"op": "stablehlo/broadcast_in_dim", "invars": [tx.id], "outvars": [out_id], "type": out_type,
           "attrs": {"broadcast_dimensions": list(bcast_dims), "target_shape": list(target_shape)}})
    return Tracer(out_id, out_type)


def slice(x, start_indices, limit_indices, strides):
    """tensor.clj:312-338 (tracer-valued bounds count as 0 / full / 1)."""
    tx = emit_constant(x, None)
    t_kw, in_shape, dtype = tx.type
    out_shape = []
    for i in range(len(in_shape)):
        s = start_indices[i] if i < len(start_indices) else 0
        l = limit_indices[i] if i < len(limit_indices) else in_shape[i]
        st = strides[i] if i < len(strides) else 1
        s_num = 0 if tracer_p(s) else int(s)
        l_num = int(in_shape[i]) if tracer_p(l) else int(l)
        st_num = 1 if tracer_p(st) else int(st)
        out_shape.append(int(math.ceil((l_num - s_num) / float(st_num))))
    out_type = (t_kw, tuple(out_shape), dtype)
    out_id = gen_var_id("t_slice")
    _emit({"op": "stablehlo/slice", "invars": [tx.id], "outvars": [out_id], "type": out_type,
           "attrs": {"start_indices": list(start_indices), "limit_indices": list(limit_indices),
                     "strides": list(strides)}})
    return Tracer(out_id, out_type)


def dynamic_update_slice(operand, update, start_indices):
    t_op = emit_constant(operand, None)
    t_up = emit_constant(update, None)
    out_id = gen_var_id("t_dus")
    _emit({"op": "stablehlo/dynamic_update_slice", "invars": [t_op.id, t_up.id], "outvars": [out_id],
           "attrs": {"start_indices": list(start_indices)}})
    return Tracer(out_id, t_op.type)


def iota(length: int, dtype: Optional[str] = None):
    dt = dtype or "i32"
    out_type = ("tensor", (int(length),), dt)
    out_id = gen_var_id("t_iota")
    _emit({"op": "stablehlo/iota", "invars": [], "outvars": [out_id],
           "attrs": {"iota_dimension": 0, "len": length, "dtype": dt}})
    return Tracer(out_id, out_type)


def gather(operand, start_indices):
    """tensor.clj:385-415 - indices reshaped to end in an index-vector dim of 1."""
    t_op = emit_constant(operand, None)
    raw_idx = emit_constant(start_indices, None)
    op_kw, op_shape, dtype = t_op.type
    idx_shape = raw_idx.type[1]
    idx_rank = len(idx_shape)
    if idx_rank == 0:
        t_idx = reshape(raw_idx, [1])
    elif idx_rank == 1:
        t_idx = reshape(raw_idx, [idx_shape[0], 1])
    elif idx_rank == 2:
        t_idx = reshape(raw_idx, [idx_shape[0], idx_shape[1], 1])
    else:
        t_idx = raw_idx
    final_rank = len(t_idx.type[1])
    hidden = op_shape[-1]
    out_shape = (hidden,) if idx_rank == 0 else tuple(idx_shape) + (hidden,)
    out_id = gen_var_id("t_gather")
    _emit({"op": "stablehlo/gather", "invars": [t_op.id, t_idx.id], "outvars": [out_id],
           "attrs": {"offset_dims": [final_rank - 1], "collapsed_slice_dims": [0], "start_index_map": [0],
                     "index_vector_dim": final_rank - 1, "slice_sizes": [1, hidden]}})
    return Tracer(out_id, (op_kw, out_shape, dtype))


def _reduce(op: str, prefix: str, x, axes, keep_dims):
    tx = emit_constant(x, None)
    t_kw, shape, dtype = tx.type
    rank = len(shape)
    norm = [rank + a if a < 0 else a for a in (axes if axes is not None else [-1])]
    aset = set(norm)
    out_shape = []
    for i, d in enumerate(shape):
        if i in aset:
            if keep_dims:
                out_shape.append(1)
        else:
            out_shape.append(d)
    out_id = gen_var_id(prefix)
    _emit({"op": op, "invars": [tx.id], "outvars": [out_id], "attrs": {"axes": norm, "keep_dims": keep_dims}})
    return Tracer(out_id, (t_kw, tuple(out_shape), dtype))


def reduce_sum(x, axes=(-1,), keep_dims=True):
    return _reduce("stablehlo/reduce_sum", "t_sum", x, list(axes), keep_dims)


def reduce_max(x, axes=(-1,), keep_dims=True):
    return _reduce("stablehlo/reduce_max", "t_max", x, list(axes), keep_dims)


def reduce_mean(x, axes=(-1,), keep_dims=True):
    """tensor.clj:467-476 - reduce_sum divided by the (double) element count."""
    tx = emit_constant(x, None)
    shape = tx.type[1]
    rank = len(shape)
    norm = [rank + a if a < 0 else a for a in axes]
    cnt = 1.0
    for a in norm:
        cnt *= shape[a]
    s = reduce_sum(tx, axes=norm, keep_dims=keep_dims)
    return div(s, float(cnt))


def compare_t(a, b, direction: str):
    return _binary("stablehlo/compare", "t_cmp", a, b, {"comparison_direction": str(direction)}, "i1")


def select(pred, on_true, on_false):
    """tensor.clj:483-515."""
    t_pred = emit_constant(pred, None)
    pred_shape = t_pred.type[1]
    t_true = emit_constant(on_true, None)
    t_false = emit_constant(on_false, t_true.type)
    t_kw, true_shape, dtype = t_true.type
    out_shape = _broadcast_shapes(pred_shape, true_shape)
    r = len(out_shape)

    def bc(t, shp):
        if tuple(shp) == out_shape:
            return t
        return broadcast_in_dim(t, out_shape, list(range(r - len(shp), r)))

    p_b = bc(t_pred, pred_shape)
    t_b = bc(t_true, true_shape)
    f_b = bc(t_false, t_false.type[1])
    out_id = gen_var_id("t_select")
    _emit({"op": "stablehlo/select", "invars": [p_b.id, t_b.id, f_b.id], "outvars": [out_id]})
    return Tracer(out_id, (t_kw, out_shape, dtype))


def eq(a, b):
    return compare_t(a, b, "EQ")


def argmax(x, axis=-1):
    """tensor.clj:519-532 - ties resolve to the HIGHEST index (max of masked iota)."""
    tx = emit_constant(x, None)
    shape = tx.type[1]
    rank = len(shape)
    ax = rank + axis if axis < 0 else axis
    n = shape[ax]
    mx = reduce_max(tx, axes=[ax], keep_dims=True)
    is_max = eq(tx, mx)
    idx_shape = [1] * rank
    idx_shape[ax] = n
    idx_const = emit_constant(list(range(n)), ("tensor", tuple(idx_shape), "i32"))
    masked = mul(convert(is_max, "i32"), idx_const)
    return reduce_max(masked, axes=[ax], keep_dims=False)


def all_reduce(x, replica_count: int, reduce: str = "sum"):
    """Sum (``reduce="sum"``) or elementwise maximum (``"max"``) of ``x`` over
    the ``replica_count`` ranks of a tensor-parallel group.

    An addition of this repository for tensor parallelism: the reference
    (clj-xla) has no multi-device code and its tensor API no collectives."""
    if reduce not in ("sum", "max"):
        raise ValueError(f"all_reduce: unsupported reduction {reduce!r}")
    tx = emit_constant(x, None)
    out_id = gen_var_id("t_allreduce")
    attrs = {"replica_count": int(replica_count)}
    if reduce == "max":
        attrs["reduce"] = "max"
    _emit({"op": "stablehlo/all_reduce", "invars": [tx.id], "outvars": [out_id], "attrs": attrs})
    return Tracer(out_id, tx.type)


def trace_graph(graph_name: str, invars, f) -> dict:
    """trace.clj:6-22 - run ``f`` on input Tracers and collect the EDN graph."""
    global _CTX
    prev = _CTX
    _CTX = _TraceCtx()
    try:
        inputs = [Tracer(name, typ) for name, typ in invars]
        res = f(*inputs)
        outs = res if isinstance(res, list) else [res]
        graph = {"name": graph_name,
                 "invars": [(name, ("tensor", tuple(t[1]), t[2])) for name, t in invars],
                 "outvars": [o.id for o in outs],
                 "eqns": _CTX.eqns}
    finally:
        _CTX = prev
    return validate_graph(graph)


def validate_graph(graph: dict) -> dict:
    """stablehlo.clj:6-34 (GraphSchema) restated as structural checks."""
    ok_dtypes = {"f32", "f64", "i32", "i64", "f16", "bf16", "i8", "i16", "u8", "u16", "u32", "u64"}
    if not isinstance(graph, dict):
        raise ValueError("Invalid SSA Graph EDN schema")
    for key in ("name", "invars", "outvars", "eqns"):
        if key not in graph:
            raise ValueError(f"Invalid SSA Graph EDN schema: missing {key}")
    if not isinstance(graph["name"], str) or not isinstance(graph["eqns"], list):
        raise ValueError("Invalid SSA Graph EDN schema")
    for name, t in graph["invars"]:
        if not isinstance(name, str) or t[0] != "tensor" or t[2] not in ok_dtypes:
            raise ValueError(f"Invalid SSA Graph EDN schema: invar {name!r}")
        if not all(isinstance(d, int) for d in t[1]):
            raise ValueError(f"Invalid SSA Graph EDN schema: invar {name!r} dims")
    for e in graph["eqns"]:
        if "op" not in e or "outvars" not in e:
            raise ValueError("Invalid SSA Graph EDN schema: equation")
    return graph
