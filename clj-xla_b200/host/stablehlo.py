"""EDN SSA graph -> StableHLO MLIR text.

Host-side mirror of ``src/clj_xla/stablehlo.clj:36-600``.  The printed text is
the semantic contract handed to the PJRT library, so this restatement keeps the
printer's behaviour exactly, including its quirks:

* result dtypes are re-inferred from the *printer's* own var-type table
  (``infer-var-types`` :70-246), not taken from the tracer; elementwise results
  take the operand type with the largest ``[rank, numel]`` (ties: last operand,
  ``find-tensor-type`` :62-68);
* operands whose dtype differs from the result get an inserted
  ``stablehlo.convert`` and scalars / low-rank operands get an inserted
  ``broadcast_in_dim`` chosen by regex (:493-551);
* float constants are printed ``%.6e`` (:263,269) and reductions start from
  ``-1.000000e+30`` (max) or ``0.000000e+00`` (:450-452);
* dynamic-update-slice start indices are converted/reshaped to scalar i32
  (:355-386).
"""
from __future__ import annotations

import re
from typing import Dict, List, Optional

_INT_DT = re.compile(r"^(?:i32|i64|i8|i1|ui8|ui32|si32)$")


def type_to_mlir(t) -> str:
    """stablehlo.clj:36-43 ``type->mlir-string``."""
    _, shape, dtype = t
    if len(shape):
        return "tensor<" + "x".join(str(int(d)) for d in shape) + "x" + dtype + ">"
    return "tensor<" + dtype + ">"


def _op_name(op: str) -> str:
    """stablehlo.clj:45-51 ``format-op-name``."""
    if op == "stablehlo/exp":
        return "stablehlo.exponential"
    ns, name = op.split("/", 1)
    if "/" in name:
        return name.replace("/", ".")
    return "stablehlo." + name


def parse_tensor_dims(type_str: Optional[str]):
    """stablehlo.clj:53-60."""
    if type_str is None:
        return None
    m = re.search(r"tensor<([0-9x]+)x([a-z0-9]+)>", type_str)
    if m:
        return [int(d) for d in m.group(1).split("x")], m.group(2)
    m = re.search(r"tensor<([a-z0-9]+)>", type_str)
    if m:
        return [], m.group(1)
    return None


def _sort_key(t):
    p = parse_tensor_dims(t)
    if p is None:
        return (0, 0)
    n = 1
    for d in p[0]:
        n *= d
    return (len(p[0]), n)


def find_tensor_type(invars, var_types) -> Optional[str]:
    """stablehlo.clj:62-68 - largest [rank, numel], last one wins on ties."""
    types = [var_types[v] for v in invars if v in var_types and var_types[v] is not None]
    if not types:
        return None
    return sorted(types, key=_sort_key)[-1]


def _tstr(dims, dtype) -> str:
    return "tensor<" + "x".join(str(d) for d in dims) + "x" + dtype + ">"


def _is_tracer_idx(idx) -> bool:
    return hasattr(idx, "id") and hasattr(idx, "type")


def _num(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def infer_var_types(invars, eqns) -> Dict[str, str]:
    """stablehlo.clj:70-246."""
    initial = {name: type_to_mlir(t) for name, t in invars}
    acc = dict(initial)
    for eqn in eqns:
        op = eqn["op"]
        in_vars = eqn.get("invars") or []
        outvars = eqn["outvars"]
        attrs = eqn.get("attrs") or {}
        non_scalar_t = find_tensor_type(in_vars, acc)
        first_in = in_vars[0] if in_vars else None
        in_type = non_scalar_t or (acc.get(first_in) if first_in is not None else None)
        out0 = outvars[0]
        if op == "stablehlo/constant":
            if eqn.get("type") is not None:
                acc[out0] = type_to_mlir(eqn["type"])
            else:
                acc[out0] = "tensor<128x128xf32>" if isinstance(eqn.get("value"), (list, tuple)) else "tensor<f32>"
        elif op == "stablehlo/gather":
            operand, idx = in_vars[0], in_vars[1]
            op_t = acc.get(operand, "tensor<50257x768xf32>")
            idx_t = acc.get(idx, "tensor<1x128xi32>")
            op_dims, op_dt = parse_tensor_dims(op_t) or ([50257, 768], "f32")
            idx_dims, _ = parse_tensor_dims(idx_t) or ([1, 128], "i32")
            hidden = op_dims[-1]
            if len(idx_dims) == 0:
                base = []
            elif len(idx_dims) == 1 and idx_dims[0] == 1:
                base = []
            elif len(idx_dims) > 1 and idx_dims[-1] == 1:
                base = idx_dims[:-1]
            else:
                base = idx_dims
            out_dims = [hidden] if not base else base + [hidden]
            acc[out0] = _tstr(out_dims, op_dt)
        elif op == "stablehlo/convert":
            tgt = attrs.get("target_dtype", "f32")
            in_dims = (parse_tensor_dims(in_type) or ([1], "i32"))[0]
            acc[out0] = _tstr(in_dims, tgt) if in_dims else "tensor<" + tgt + ">"
        elif op == "stablehlo/compare":
            t = acc.get(in_vars[0], "tensor<1x128x768xf32>")
            in_dims = (parse_tensor_dims(t) or ([1], "f32"))[0]
            acc[out0] = _tstr(in_dims, "i1") if in_dims else "tensor<i1>"
        elif op == "stablehlo/reshape":
            new_shape = attrs.get("shape", [1, 128, 1])
            in_dt = (parse_tensor_dims(in_type) or ([1, 128], "f32"))[1]
            acc[out0] = _tstr(new_shape, in_dt) if len(new_shape) else "tensor<" + in_dt + ">"
        elif op == "stablehlo/transpose":
            perm = attrs.get("permutation", [0, 2, 1])
            in_dims, in_dt = parse_tensor_dims(in_type) or ([1, 128, 768], "f32")
            acc[out0] = _tstr([in_dims[p] for p in perm], in_dt)
        elif op == "stablehlo/broadcast_in_dim":
            ts = attrs.get("target_shape", [1, 3, 3, 128, 64])
            in_dt = (parse_tensor_dims(in_type) or ([1, 3, 1, 128, 64], "f32"))[1]
            acc[out0] = _tstr(ts, in_dt) if len(ts) else "tensor<" + in_dt + ">"
        elif op == "stablehlo/custom_call":
            acc[out0] = acc.get(in_vars[0] if in_vars else None, "tensor<1xi32>")
        elif op == "stablehlo/dynamic_update_slice":
            acc[out0] = acc.get(in_vars[0], "tensor<1x1x4096x256xbf16>")
        elif op == "stablehlo/dynamic_slice":
            sizes = attrs.get("slice_sizes", [1, 1, 4096, 256])
            in_dt = (parse_tensor_dims(in_type) or ([1, 1, 4096, 256], "f32"))[1]
            acc[out0] = _tstr(sizes, in_dt)
        elif op == "stablehlo/slice":
            starts = attrs.get("start_indices", [0, 0, 0])
            limits = attrs.get("limit_indices", [1, 128, 768])
            strides = attrs.get("strides", [1, 1, 1])
            in_dims, in_dt = parse_tensor_dims(in_type) or ([1, 128, 2304], "f32")
            out = []
            for i in range(len(in_dims)):
                s = starts[i] if i < len(starts) else 0
                l = limits[i] if i < len(limits) else in_dims[i]
                st = strides[i] if i < len(strides) else 1
                sv = int(s) if _num(s) else 0
                lv = int(l) if _num(l) else int(in_dims[i])
                stv = int(st) if _num(st) else 1
                out.append(int(-(-(lv - sv) // stv)) if stv > 0 else 0)
            acc[out0] = _tstr(out, in_dt)
        elif op == "stablehlo/concatenate":
            in_types = [acc.get(v, "tensor<1x8x128x64xf32>") for v in in_vars]
            dims, dt = parse_tensor_dims(in_types[0]) or ([1, 8, 128, 64], "f32")
            dim = attrs.get("dimension", 3)
            di = len(dims) + dim if dim < 0 else dim
            total = 0
            for t in in_types:
                d = (parse_tensor_dims(t) or (dims, "f32"))[0]
                total += d[di]
            od = list(dims)
            od[di] = total
            acc[out0] = _tstr(od, dt)
        elif op in ("stablehlo/reduce_mean", "stablehlo/reduce_sum", "stablehlo/reduce_max"):
            axes = attrs.get("axes", [2])
            keep = attrs.get("keep_dims", True)
            in_dims, in_dt = parse_tensor_dims(in_type) or ([1, 128, 768], "f32")
            rank = len(in_dims)
            na = set(rank + a if a < 0 else a for a in axes)
            out = []
            for i, d in enumerate(in_dims):
                if i in na:
                    if keep:
                        out.append(1)
                else:
                    out.append(d)
            acc[out0] = "tensor<" + "x".join(str(d) for d in out) + "x" + in_dt + ">"
        elif op == "stablehlo/dot_general":
            lhs_t = acc.get(in_vars[0], "tensor<1x128x768xf32>")
            rhs_t = acc.get(in_vars[1], "tensor<768x50257xf32>")
            ld, ldt = parse_tensor_dims(lhs_t) or ([1, 128, 768], "f32")
            rd, _ = parse_tensor_dims(rhs_t) or ([768, 50257], "f32")
            cd = attrs.get("contracting_dims") or {}
            bd = attrs.get("batch_dims") or {}
            cl = set(cd.get("lhs", [len(ld) - 1]))
            cr = set(cd.get("rhs", [0]))
            bl = set(bd.get("lhs", []))
            br = set(bd.get("rhs", []))
            batch = [ld[i] for i in bd.get("lhs", [])]
            lf = [d for i, d in enumerate(ld) if i not in cl and i not in bl]
            rf = [d for i, d in enumerate(rd) if i not in cr and i not in br]
            acc[out0] = _tstr(batch + lf + rf, ldt)
        elif op == "stablehlo/iota":
            acc[out0] = "tensor<" + str(attrs.get("len", 128)) + "x" + attrs.get("dtype", "i32") + ">"
        else:
            target = in_type or "tensor<1x128x768xf32>"
            for v in outvars:
                if v not in initial:
                    acc[v] = target
    return acc


def _fmt_float(v) -> str:
    return "%.6e" % float(v)


def _flatten(v):
    if isinstance(v, (list, tuple)):
        for x in v:
            yield from _flatten(x)
    else:
        yield v


_BC_SCALAR = re.compile(r"^tensor<(?:bf16|f16|f32|f64|i8|i32|i64)>$")
_BC_RANK1 = re.compile(r"^tensor<\d+x(?:bf16|f16|f32|f64|i8|i32|i64)>$")
_BC_1N1 = re.compile(r"^tensor<1x\d+x1x(?:bf16|f16|f32|f64|i8|i32|i64)>$")
_BC_1NNN = re.compile(r"^tensor<1x\d+x\d+x\d+x(?:bf16|f16|f32|f64|i8|i32|i64)>$")
_BC_11NN = re.compile(r"^tensor<1x1x\d+x\d+x(?:bf16|f16|f32|f64|i8|i32|i64)>$")
_BC_NN = re.compile(r"^tensor<\d+x\d+x(?:bf16|f16|f32|f64|i8|i32|i64)>$")
_OUT_DIMS = re.compile(r"tensor<([0-9x]+)x(?:bf16|f16|f32|f64|i8|i32|i64)>")


def _dus_index_lines(out_var, prefix, starts, var_types):
    lines, args = [], []
    for i, idx in enumerate(starts):
        c_var = f"{out_var}_{prefix}{i}"
        if _is_tracer_idx(idx) or isinstance(idx, str):
            v_id = idx.id if _is_tracer_idx(idx) else idx
            v_type = var_types.get(v_id, "tensor<1xi32>")
            v_dims = (parse_tensor_dims(v_type) or ([1], "i32"))[0]
            if v_dims:
                v1d = _tstr(v_dims, "i32")
                lines.append(f'    %{c_var}_1d = "stablehlo.convert"(%{v_id}) : ({v_type}) -> {v1d}\n'
                             f"    %{c_var} = stablehlo.reshape %{c_var}_1d : ({v1d}) -> tensor<i32>")
            else:
                lines.append(f'    %{c_var} = "stablehlo.convert"(%{v_id}) : ({v_type}) -> tensor<i32>')
        else:
            lines.append(f"    %{c_var} = stablehlo.constant dense<{int(idx)}> : tensor<i32>")
        args.append(f"%{c_var}")
    return lines, args


def format_equation(eqn: dict, var_types: Dict[str, str]) -> str:
    """stablehlo.clj:248-580."""
    op = eqn["op"]
    invars = eqn.get("invars") or []
    outvars = eqn["outvars"]
    attrs = eqn.get("attrs") or {}
    value = eqn.get("value")
    mlir_op = _op_name(op)
    out = outvars[0]
    if op == "stablehlo/constant":
        out_type = var_types.get(out, "tensor<f32>")
        dt = (parse_tensor_dims(out_type) or (None, None))[1] or "f32"
        is_int = bool(_INT_DT.match(dt))
        if isinstance(value, (list, tuple)):
            flat = list(_flatten(value))
            if is_int:
                vals = [str(int(v)) if _num(v) else "0" for v in flat]
            else:
                vals = [_fmt_float(v) if _num(v) else "0.000000e+00" for v in flat]
            t1d = f"tensor<{len(flat)}x{dt}>"
            return (f"    %{out}_1d = {mlir_op} dense<[{', '.join(vals)}]> : {t1d}\n"
                    f"    %{out} = stablehlo.reshape %{out}_1d : ({t1d}) -> {out_type}")
        v = value if value is not None else (0 if is_int else 0.0)
        num = str(int(v)) if is_int else _fmt_float(v)
        return f"    %{out} = {mlir_op} dense<{num}> : {out_type}"
    if op == "stablehlo/convert":
        in_var = invars[0]
        in_type = var_types.get(in_var, "tensor<1x128x768xf32>")
        tgt = attrs.get("target_dtype", "f32")
        in_dims = (parse_tensor_dims(in_type) or ([1], "i32"))[0]
        out_type = _tstr(in_dims, tgt) if in_dims else f"tensor<{tgt}>"
        return f'    %{out} = "stablehlo.convert"(%{in_var}) : ({in_type}) -> {out_type}'
    if op == "stablehlo/compare":
        a, b = invars[0], invars[1]
        at = var_types.get(a, "tensor<1x128x768xf32>")
        bt = var_types.get(b, at)
        ot = var_types.get(out, "tensor<1x128x768xi1>")
        d = attrs.get("comparison_direction", "EQ")
        return (f'    %{out} = "stablehlo.compare"(%{a}, %{b}) {{comparison_direction = '
                f"#stablehlo<comparison_direction {d}>}} : ({at}, {bt}) -> {ot}")
    if op == "stablehlo/select":
        p, t, f = invars
        pt = var_types.get(p, "tensor<1x128x768xi1>")
        tt = var_types.get(t, "tensor<1x128x768xf32>")
        ft = var_types.get(f, tt)
        ot = var_types.get(out, tt)
        return f'    %{out} = "stablehlo.select"(%{p}, %{t}, %{f}) : ({pt}, {tt}, {ft}) -> {ot}'
    if op == "stablehlo/gather":
        operand, idx = invars
        ot_ = var_types.get(operand, "tensor<50257x768xf32>")
        it = var_types.get(idx, "tensor<1x128xi32>")
        rt = var_types.get(out, "tensor<1x128x768xf32>")
        j = lambda xs: ", ".join(str(x) for x in xs)
        return (f'    %{out} = "stablehlo.gather"(%{operand}, %{idx}) {{dimension_numbers = #stablehlo.gather<'
                f"offset_dims = [{j(attrs.get('offset_dims', [2]))}], "
                f"collapsed_slice_dims = [{j(attrs.get('collapsed_slice_dims', [0]))}], "
                f"start_index_map = [{j(attrs.get('start_index_map', [0]))}], "
                f"index_vector_dim = {attrs.get('index_vector_dim', 2)}>, "
                f"slice_sizes = array<i64: {j(attrs.get('slice_sizes', [1, 768]))}>, "
                f"indices_are_sorted = false}} : ({ot_}, {it}) -> {rt}")
    if op == "stablehlo/reshape":
        iv = invars[0]
        it = var_types.get(iv, "tensor<1x128xf32>")
        ot = var_types.get(out, "tensor<1x128x1xf32>")
        return f"    %{out} = stablehlo.reshape %{iv} : ({it}) -> {ot}"
    if op == "stablehlo/transpose":
        iv = invars[0]
        it = var_types.get(iv, "tensor<1x128x768xf32>")
        ot = var_types.get(out, "tensor<1x768x128xf32>")
        perm = ", ".join(str(p) for p in attrs.get("permutation", [0, 2, 1]))
        return f'    %{out} = "stablehlo.transpose"(%{iv}) {{permutation = array<i64: {perm}>}} : ({it}) -> {ot}'
    if op == "stablehlo/broadcast_in_dim":
        iv = invars[0]
        it = var_types.get(iv, "tensor<1x3x1x128x64xf32>")
        ot = var_types.get(out, "tensor<1x3x3x128x64xf32>")
        bd = attrs.get("broadcast_dimensions", [0, 1, 2, 3, 4])
        ba = ("array<i64: " + ", ".join(str(x) for x in bd) + ">") if len(bd) else "array<i64>"
        return f'    %{out} = "stablehlo.broadcast_in_dim"(%{iv}) {{broadcast_dimensions = {ba}}} : ({it}) -> {ot}'
    if op == "stablehlo/slice":
        iv = invars[0]
        it = var_types.get(iv, "tensor<1x128x2304xf32>")
        ot = var_types.get(out, "tensor<1x128x768xf32>")
        st = ", ".join(str(int(x)) if _num(x) else "0" for x in attrs.get("start_indices", [0, 0, 0]))
        li = ", ".join(str(int(x)) if _num(x) else "1" for x in attrs.get("limit_indices", [1, 128, 768]))
        sr = ", ".join(str(int(x)) if _num(x) else "1" for x in attrs.get("strides", [1, 1, 1]))
        return (f'    %{out} = "stablehlo.slice"(%{iv}) {{limit_indices = array<i64: {li}>, '
                f"start_indices = array<i64: {st}>, strides = array<i64: {sr}>}} : ({it}) -> {ot}")
    if op == "stablehlo/dynamic_update_slice":
        opv, upv = invars[0], invars[1]
        opt = var_types.get(opv, "tensor<1x4x128x256xf32>")
        upt = var_types.get(upv, "tensor<1x4x1x256xf32>")
        ot = var_types.get(out, opt)
        starts = attrs.get("start_indices", [0, 0, 0, 0])
        in_dims = (parse_tensor_dims(opt) or ([1, 4, 128, 256], "f32"))[0]
        rank = len(in_dims)
        lines, args = _dus_index_lines(out, "c", list(starts)[:rank], var_types)
        line = (f'    %{out} = "stablehlo.dynamic_update_slice"(%{opv}, %{upv}, {", ".join(args)}) : ('
                f"{opt}, {upt}, {', '.join(['tensor<i32>'] * rank)}) -> {ot}")
        return "\n".join(lines + [line])
    if op == "stablehlo/dynamic_slice":
        opv = invars[0]
        opt = var_types.get(opv, "tensor<1x1x12288x256xf32>")
        ot = var_types.get(out, opt)
        sizes = attrs.get("slice_sizes", [1, 1, 12288, 256])
        starts = attrs.get("start_indices", [0, 0, 0, 0])
        in_dims = (parse_tensor_dims(opt) or ([1, 1, 12288, 256], "f32"))[0]
        rank = len(in_dims)
        lines, args = _dus_index_lines(out, "s", list(starts)[:rank], var_types)
        line = (f'    %{out} = "stablehlo.dynamic_slice"(%{opv}, {", ".join(args)}) {{slice_sizes = array<i64: '
                f"{', '.join(str(s) for s in sizes)}>}} : ({opt}, {', '.join(['tensor<i32>'] * rank)}) -> {ot}")
        return "\n".join(lines + [line])
    if op == "stablehlo/iota":
        ln = attrs.get("len", 128)
        dt = attrs.get("dtype", "i32")
        dim = attrs.get("iota_dimension", 0)
        return f'    %{out} = "stablehlo.iota"() {{iota_dimension = {dim} : i64}} : () -> tensor<{ln}x{dt}>'
    if op == "stablehlo/concatenate":
        args = ", ".join("%" + v for v in invars)
        tys = ", ".join(var_types.get(v, "tensor<1x8x128x64xf32>") for v in invars)
        ot = var_types.get(out, "tensor<1x8x128x128xf32>")
        return f'    %{out} = "stablehlo.concatenate"({args}) {{dimension = {attrs.get("dimension", 3)} : i64}} : ({tys}) -> {ot}'
    if op in ("stablehlo/reduce_mean", "stablehlo/reduce_sum", "stablehlo/reduce_max"):
        iv = invars[0]
        it = var_types.get(iv, "tensor<f32>")
        ot = var_types.get(out, "tensor<1x128x1xf32>")
        in_dims, in_dt = parse_tensor_dims(it) or ([1, 12, 128, 128], "f32")
        rank = len(in_dims)
        axes = attrs.get("axes", [rank - 1])
        na = [rank + a if a < 0 else a for a in axes]
        red = "stablehlo.maximum" if op == "stablehlo/reduce_max" else "stablehlo.add"
        is_int = bool(_INT_DT.match(str(in_dt)))
        if op == "stablehlo/reduce_max":
            init = "0" if is_int else "-1.000000e+30"
        else:
            init = "0" if is_int else "0.000000e+00"
        nset = set(na)
        rdims = [in_dims[i] for i in range(rank) if i not in nset]
        rt = _tstr(rdims, in_dt) if rdims else f"tensor<{in_dt}>"
        return (f"    %{out}_c0 = stablehlo.constant dense<{init}> : tensor<{in_dt}>\n"
                f'    %{out}_red = "stablehlo.reduce"(%{iv}, %{out}_c0) ({{\n'
                f"    ^bb0(%arg_a: tensor<{in_dt}>, %arg_b: tensor<{in_dt}>):\n"
                f"      %arg_res = {red} %arg_a, %arg_b : tensor<{in_dt}>\n"
                f'      "stablehlo.return"(%arg_res) : (tensor<{in_dt}>) -> ()\n'
                f"    }}) {{dimensions = array<i64: {', '.join(str(a) for a in na)}>}} : ({it}, tensor<{in_dt}>) -> {rt}\n"
                f"    %{out} = stablehlo.reshape %{out}_red : ({rt}) -> {ot}")
    if op == "stablehlo/all_reduce":
        # tensor-parallel partial sums; an addition of this repository (the
        # reference prints no collectives: clj-xla runs on one device)
        iv = invars[0]
        it = var_types.get(iv, "tensor<f32>")
        _, dt = parse_tensor_dims(it)
        n = int(attrs["replica_count"])
        ranks = ", ".join(str(i) for i in range(n))
        body = "stablehlo.maximum" if attrs.get("reduce") == "max" else "stablehlo.add"
        return (f'    %{out} = "stablehlo.all_reduce"(%{iv}) ({{\n'
                f"    ^bb0(%arg_a: tensor<{dt}>, %arg_b: tensor<{dt}>):\n"
                f"      %arg_res = {body} %arg_a, %arg_b : tensor<{dt}>\n"
                f'      "stablehlo.return"(%arg_res) : (tensor<{dt}>) -> ()\n'
                f"    }}) {{replica_groups = dense<[[{ranks}]]> : tensor<1x{n}xi64>}} : ({it}) -> {it}")
    if op == "stablehlo/dot_general":
        lhs, rhs = invars
        lt = var_types.get(lhs, "tensor<1x128x768xf32>")
        rt = var_types.get(rhs, "tensor<768x50257xf32>")
        ot = var_types.get(out, "tensor<1x128x50257xf32>")
        cd = attrs.get("contracting_dims") or {}
        bd = attrs.get("batch_dims") or {}
        lc = cd.get("lhs", [2] if re.search(r"tensor<\d+x\d+x\d+x?", lt) else [1])
        rc = cd.get("rhs", [0])
        lb = bd.get("lhs")
        rb = bd.get("rhs")
        j = lambda xs: ", ".join(str(x) for x in xs)
        da = "#stablehlo.dot<"
        if lb:
            da += f"lhs_batching_dimensions = [{j(lb)}], "
        if rb:
            da += f"rhs_batching_dimensions = [{j(rb)}], "
        da += f"lhs_contracting_dimensions = [{j(lc)}], rhs_contracting_dimensions = [{j(rc)}]>"
        return (f'    %{out} = "stablehlo.dot_general"(%{lhs}, %{rhs}) {{dot_dimension_numbers = {da}, '
                f"precision = [#stablehlo<precision DEFAULT>, #stablehlo<precision DEFAULT>]}} : ({lt}, {rt}) -> {ot}")
    # generic elementwise form with implicit converts / broadcasts (:493-580)
    in_types = [var_types.get(v, "tensor<1x128x768xf32>") for v in invars]
    out_type = var_types.get(out) or find_tensor_type(invars, var_types) or \
        var_types.get(invars[0] if invars else None) or "tensor<1x128x768xf32>"
    out_dt = (parse_tensor_dims(out_type) or ([1], "f32"))[1]
    prep: List[str] = []

    def add_line(l):
        if l not in prep:
            prep.append(l)

    vstrs = []
    for inv, raw in zip(invars, in_types):
        in_dims, in_dt = parse_tensor_dims(raw) or ([1], "f32")
        name, in_t = inv, raw
        if in_dt != out_dt and raw != out_type:
            c_var = f"{inv}_conv_{out}"
            target = _tstr(in_dims, out_dt) if in_dims else f"tensor<{out_dt}>"
            add_line(f'    %{c_var} = "stablehlo.convert"(%{inv}) : ({raw}) -> {target}')
            name, in_t = c_var, target
        if in_t == out_type:
            vstrs.append("%" + name)
            continue
        bvar = f"{name}_bcast_{out}"
        if _BC_SCALAR.match(in_t):
            add_line(f'    %{bvar} = "stablehlo.broadcast_in_dim"(%{name}) {{broadcast_dimensions = array<i64>}} : ({in_t}) -> {out_type}')
            vstrs.append("%" + bvar)
        elif _BC_RANK1.match(in_t):
            m = _OUT_DIMS.search(out_type)
            ods = m.group(1) if m else ""
            bdim = max(0, len(ods.split("x")) - 1)
            add_line(f'    %{bvar} = "stablehlo.broadcast_in_dim"(%{name}) {{broadcast_dimensions = array<i64: {bdim}>}} : ({in_t}) -> {out_type}')
            vstrs.append("%" + bvar)
        elif _BC_1N1.match(in_t):
            add_line(f'    %{bvar} = "stablehlo.broadcast_in_dim"(%{name}) {{broadcast_dimensions = array<i64: 0, 1, 2>}} : ({in_t}) -> {out_type}')
            vstrs.append("%" + bvar)
        elif _BC_1NNN.match(in_t) or _BC_11NN.match(in_t):
            add_line(f'    %{bvar} = "stablehlo.broadcast_in_dim"(%{name}) {{broadcast_dimensions = array<i64: 0, 1, 2, 3>}} : ({in_t}) -> {out_type}')
            vstrs.append("%" + bvar)
        elif _BC_NN.match(in_t):
            add_line(f'    %{bvar} = "stablehlo.broadcast_in_dim"(%{name}) {{broadcast_dimensions = array<i64: 2, 3>}} : ({in_t}) -> {out_type}')
            vstrs.append("%" + bvar)
        else:
            vstrs.append("%" + name)
    meta = eqn.get("metadata") or {}
    loc = f' loc("{meta["op-name"]}")' if meta.get("op-name") else ""
    if op == "stablehlo/custom_call":
        iv = invars[0]
        tgt = attrs.get("call_target_name", "copy")
        it = var_types.get(iv, "tensor<1xi32>")
        ot = var_types.get(out, it)
        raw_line = f'    %{out} = "stablehlo.custom_call"(%{iv}) {{call_target_name = "{tgt}"}} : ({it}) -> {ot}'
    else:
        raw_line = f"    %{out} = {mlir_op} {', '.join(vstrs)} : {out_type}"
    return "\n".join(prep + [raw_line + loc])


def graph_to_mlir_text(graph: dict) -> str:
    """stablehlo.clj:582-600 ``graph->mlir-text``."""
    from .tensor import validate_graph
    validate_graph(graph)
    name = graph["name"]
    invars = graph["invars"]
    outvars = graph["outvars"]
    eqns = graph["eqns"]
    vt = infer_var_types(invars, eqns)
    params = ", ".join(f"%{v}: {type_to_mlir(t)}" for v, t in invars)
    rtypes = [vt.get(v, "tensor<f32>") for v in outvars]
    lines = [format_equation(e, vt) for e in eqns]
    return (f"module @{name} {{\n"
            f"  func.func @main({params}) -> ({', '.join(rtypes)}) {{\n"
            + "\n".join(lines) + "\n"
            f"    return {', '.join('%' + v for v in outvars)} : {', '.join(rtypes)}\n"
            "  }\n"
            "}\n")
