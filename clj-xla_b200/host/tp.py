"""Tensor-parallel decoding over several B200 clients, one process per GPU.

An addition of this repository: the reference runs every graph on one device
(``src/clj_xla/core.clj:129-167`` creates a single client).  Each rank traces
the shard graph of :func:`drivers.shard_config` (heads and MLP width divided by
the rank count, an ``all_reduce`` after the attention and MLP row-split
projections, ``models.py``) and runs it on its own client.  The clients of a
group share one NCCL communicator: rank 0 makes the id through the library
(``cljxla_b200_nccl_unique_id``), the host passes it to every rank, and each
client is created with ``tp_size`` / ``tp_rank`` / ``tp_nccl_id``; the graph's
all-reduces then run as NCCL all-reduces on the client's stream, inside the
executable's CUDA graph.

The greedy loop mirrors ``run-autoregressive-decode``
(``scripts/gemma4_inference.clj:399-470``): prefill, then one decode step per
token with the K/V caches kept on the device, host argmax (lowest index on
ties).  Every rank computes the same all-reduced logits, so every rank picks
the same token without a host exchange.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import core
from . import drivers as d
from .pjrt import DTYPE_ENUM
from .stablehlo import graph_to_mlir_text


class GroupError(RuntimeError):
    """A tensor-parallel group could not be formed; raised on every rank."""


def share_nccl_id(lib_path: Optional[str] = None) -> str:
    """Rank 0's NCCL id, broadcast over the default torch.distributed group
    (any backend: the id is host data).  If rank 0 cannot make one (NCCL not
    loadable, no network interface for its bootstrap), the failure is what
    gets broadcast, so every rank raises GroupError instead of the others
    waiting in the collective client creation for a rank that never joins."""
    import torch.distributed as dist
    obj = [None]
    if dist.get_rank() == 0:
        try:
            obj = [("ok", core.nccl_unique_id(lib_path))]
        except Exception as e:  # noqa: BLE001 - reported to every rank
            obj = [("error", f"rank 0 could not create the NCCL id: {e}")]
    dist.broadcast_object_list(obj, src=0)
    status, value = obj[0]
    if status != "ok":
        raise GroupError(value)
    return value


def setup_p2p(ctx: core.Context, slot_bytes: int = 32 << 10):
    """Switches the group's small all_reduce ops to the one-shot peer kernel:
    handles exchanged over the default torch.distributed group (a collective)."""
    import torch.distributed as dist
    hs = [None] * dist.get_world_size()
    dist.all_gather_object(hs, core.p2p_export(ctx, slot_bytes))
    core.p2p_import(ctx, hs)


def join_group(device: Optional[int] = None, lib_path: Optional[str] = None) -> core.Context:
    """Client of this process's rank in a group spanning the default
    torch.distributed group (a collective: every rank calls it)."""
    import torch.distributed as dist
    nid = share_nccl_id(lib_path)
    return core.init_tp_backend(dist.get_world_size(), dist.get_rank(), nid, device, lib_path)


def shard_graphs(cfg_full: d.ModelConfig, tp: int, batch: int, prompt_len: int, max_seq: int,
                 dynamic_prefill: bool = False) -> Tuple[d.ModelConfig, dict, dict]:
    """(per-rank config, prefill graph, decode graph) of a ``tp``-way shard."""
    cfg = d.shard_config(cfg_full, tp)
    gp = d.build_graph(cfg, "prefill", batch, prompt_len, max_seq, dynamic_prefill=dynamic_prefill)
    gd = d.build_graph(cfg, "decode", batch, prompt_len, max_seq)
    return cfg, gp, gd


def greedy_generate(ctx: core.Context, cfg: d.ModelConfig, g_pre: dict, g_dec: dict,
                    weights: Sequence[np.ndarray], prompt: np.ndarray, max_seq: int,
                    steps: int) -> Tuple[List[List[int]], List[np.ndarray]]:
    """Greedy decoding of ``steps`` tokens per batch row after ``prompt``
    [B, S] (int32).  ``weights`` are this rank's (sharded) weights in invar
    order.  Returns (tokens per row, [prefill logits, decode logits...]) with
    f32 logits as numpy arrays."""
    api = ctx["api"]
    B, S = prompt.shape
    wdt = DTYPE_ENUM[cfg.dtype]
    specs = d.weight_specs(cfg)
    ex_pre = core.compile_mlir_text(ctx, graph_to_mlir_text(g_pre), g_pre)
    ex_dec = core.compile_mlir_text(ctx, graph_to_mlir_text(g_dec), g_dec)
    wbufs = [core.buffer_from_host_buffer(ctx, w, shp, wdt) for w, (_, shp, _) in zip(weights, specs)]
    cache = d.zero_cache(cfg, B, max_seq)
    kv = [core.buffer_from_host_buffer(ctx, cache, list(cache.shape), wdt) for _ in range(2 * cfg.layers)]
    logits_all: List[np.ndarray] = []
    tokens: List[List[int]] = [[] for _ in range(B)]
    try:
        xb = core.buffer_from_host_buffer(ctx, np.ascontiguousarray(prompt, np.int32), [B, S], 4)
        pb = core.buffer_from_host_buffer(ctx, d.pos_inputs(cfg, "prefill", B, 0, S), [S], 4)
        outs = api.execute_executable(ex_pre["handle"], [xb, pb] + wbufs + kv, len(g_pre["outvars"]))
        for b in [xb, pb] + kv:
            api.destroy_buffer(b)
        kv = outs[1:]
        lg = core.buffer_to_numpy(ctx, outs[0], [B, S, cfg.vocab], "f32")
        api.destroy_buffer(outs[0])
        logits_all.append(lg)
        nxt = [d.argmax_host(lg[r, S - 1]) for r in range(B)]
        for step in range(steps):
            for r in range(B):
                tokens[r].append(nxt[r])
            if step == steps - 1:
                break
            xb = core.buffer_from_host_buffer(ctx, np.array(nxt, np.int32).reshape(B, 1), [B, 1], 4)
            pb = core.buffer_from_host_buffer(ctx, d.pos_inputs(cfg, "decode", B, S + step, 1), [1], 4)
            outs = api.execute_executable(ex_dec["handle"], [xb, pb] + wbufs + kv, len(g_dec["outvars"]))
            for b in [xb, pb] + kv:
                api.destroy_buffer(b)
            kv = outs[1:]
            lg = core.buffer_to_numpy(ctx, outs[0], [B, 1, cfg.vocab], "f32")
            api.destroy_buffer(outs[0])
            logits_all.append(lg)
            nxt = [d.argmax_host(lg[r, 0]) for r in range(B)]
    finally:
        for b in kv + wbufs:
            api.destroy_buffer(b)
    return tokens, logits_all


def oracle_generate(cfg_full: d.ModelConfig, tp: int, weights_full: Sequence[np.ndarray], prompt: np.ndarray,
                    max_seq: int, steps: int, run_tp, run_one) -> Tuple[List[List[int]], List[np.ndarray]]:
    """The same greedy loop on a CPU executor of the printed graphs:
    ``run_tp(texts, inputs_per_rank)`` for tp > 1, ``run_one(text, inputs)``
    for tp == 1 (test infrastructure passes the oracle's entry points)."""
    B, S = prompt.shape
    cfg, gp, gd = shard_graphs(cfg_full, tp, B, S, max_seq)
    tpre, tdec = graph_to_mlir_text(gp), graph_to_mlir_text(gd)
    ws = [d.shard_weights(cfg_full, list(weights_full), r, tp) for r in range(tp)]
    kv = [[d.zero_cache(cfg, B, max_seq) for _ in range(2 * cfg.layers)] for _ in range(tp)]

    def run(text, per_rank_inputs):
        if tp == 1:
            return [run_one(text, per_rank_inputs[0])]
        return run_tp([text] * tp, per_rank_inputs)

    outs = run(tpre, [[prompt.astype(np.int32), d.pos_inputs(cfg, "prefill", B, 0, S)] + ws[r] + kv[r]
                      for r in range(tp)])
    kv = [o[1:] for o in outs]
    logits_all = [np.asarray(outs[0][0], np.float32)]
    nxt = [d.argmax_host(logits_all[-1][r, S - 1]) for r in range(B)]
    tokens: List[List[int]] = [[] for _ in range(B)]
    for step in range(steps):
        for r in range(B):
            tokens[r].append(nxt[r])
        if step == steps - 1:
            break
        x = np.array(nxt, np.int32).reshape(B, 1)
        outs = run(tdec, [[x, d.pos_inputs(cfg, "decode", B, S + step, 1)] + ws[r] + kv[r] for r in range(tp)])
        kv = [o[1:] for o in outs]
        logits_all.append(np.asarray(outs[0][0], np.float32))
        nxt = [d.argmax_host(logits_all[-1][r, 0]) for r in range(B)]
    return tokens, logits_all
