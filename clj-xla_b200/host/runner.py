"""Convenience layer over :mod:`core`: run a traced graph end to end.

Uploads numpy inputs with the invar dtypes (bf16 as uint16 bit patterns),
executes, reads every result back as numpy and destroys the device buffers.
"""
from __future__ import annotations

from typing import List, Sequence

import numpy as np

from . import core
from .pjrt import DTYPE_ENUM
from .stablehlo import graph_to_mlir_text, infer_var_types, parse_tensor_dims


def out_specs(graph: dict):
    vt = infer_var_types(graph["invars"], graph["eqns"])
    specs = []
    for v in graph["outvars"]:
        dims, dt = parse_tensor_dims(vt[v])
        specs.append((tuple(dims), dt))
    return specs


def upload(ctx, graph: dict, inputs: Sequence[np.ndarray]) -> List[int]:
    bufs = []
    for (name, (_, shape, dt)), x in zip(graph["invars"], inputs):
        a = np.asarray(x)
        if dt == "bf16" and a.dtype != np.uint16:
            raise TypeError(f"bf16 input {name} must be given as uint16 bit patterns")
        bufs.append(core.buffer_from_host_buffer(ctx, a, shape, DTYPE_ENUM[dt]))
    return bufs


def run_graph(ctx, graph: dict, inputs: Sequence[np.ndarray], text: str = None) -> List[np.ndarray]:
    exe = core.compile_mlir_text(ctx, text or graph_to_mlir_text(graph), graph)
    bufs = upload(ctx, graph, inputs)
    try:
        outs = ctx["api"].execute_executable(exe["handle"], bufs, len(graph["outvars"]))
        outs = outs if isinstance(outs, list) else [outs]
        res = []
        for b, (shape, dt) in zip(outs, out_specs(graph)):
            res.append(core.buffer_to_numpy(ctx, b, shape, dt))
            core.destroy_buffer(ctx, b)
        return res
    finally:
        for b in bufs:
            core.destroy_buffer(ctx, b)
