"""Model configs, graph I/O layout and synthetic inputs for the decoder path.

Host-side mirror of the reference inference drivers: the invar order and the
prefill / decode trace functions of ``scripts/gemma2_inference.clj:172-270``,
``scripts/gemma3_inference.clj:174-284`` and ``scripts/gpt2_inference.clj:123-159``.

Graph I/O contract (same as the reference drivers):
  invars  = [x, pos, <embedding / final-norm / per-layer weights>, k_cache_0, v_cache_0, ...]
  outvars = [logits_f32, k_0, v_0, k_1, v_1, ...]

Differences from the reference drivers, all opt-in through arguments:
* ``batch`` > 1 (the reference drivers only trace batch 1; the model code is
  batch-generic);
* Gemma-2 attention softcap / alternating local windows and Gemma-3 local
  windows are passed through the layer maps;
* ``dynamic_prefill=True`` traces the prefill with tracer-valued positions
  (on-device RoPE angles and iota mask, as the decode graph already does)
  instead of the static path that embeds S*S mask and S*hd RoPE literals per
  layer - at S >= 2048 those literals are gigabytes of MLIR text.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional

import numpy as np

from . import tensor as t
from .models import full_gemma_forward, full_gpt2_forward


@dataclass(frozen=True)
class ModelConfig:
    family: str                 # "gpt2" | "gemma2" | "gemma3"
    vocab: int
    d_model: int
    layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    mlp: int
    dtype: str = "bf16"
    attn_softcap: Optional[float] = None
    final_softcap: Optional[float] = None
    window: Optional[int] = None          # local attention window
    n_positions: int = 1024               # GPT-2 learned position table
    tp: int = 1                           # tensor-parallel ranks this (per-rank) config is a shard of
    # vocab-split LM head (greedy graphs of a tensor-parallel Gemma): this rank's
    # index; its logits cover vocabulary rows [rank * V / tp, (rank + 1) * V / tp)
    vocab_rank: Optional[int] = None

    def is_local(self, i: int) -> bool:
        if self.window is None:
            return False
        if self.family == "gemma2":
            return i % 2 == 0
        if self.family == "gemma3":
            return (i + 1) % 6 != 0
        return False

    def theta(self, i: int) -> float:
        if self.family == "gemma3":
            return 1000000.0 if (i + 1) % 6 == 0 else 10000.0
        return 10000.0


GPT2_SMALL = ModelConfig("gpt2", 50257, 768, 12, 12, 12, 64, 3072, dtype="f32")
GEMMA2_2B = ModelConfig("gemma2", 256000, 2304, 26, 8, 4, 256, 9216, attn_softcap=50.0, final_softcap=30.0,
                        window=4096)
GEMMA3_4B = ModelConfig("gemma3", 262144, 2560, 34, 8, 4, 256, 10240, window=1024)
GEMMA3_12B = ModelConfig("gemma3", 262144, 3840, 48, 16, 8, 256, 15360, window=1024)
GEMMA3_27B = ModelConfig("gemma3", 262144, 5376, 62, 32, 16, 128, 21504, window=1024)

CONFIGS: Dict[str, ModelConfig] = {
    "gpt2-small": GPT2_SMALL, "gemma2-2b": GEMMA2_2B, "gemma3-4b": GEMMA3_4B,
    "gemma3-12b": GEMMA3_12B, "gemma3-27b": GEMMA3_27B,
}


def round_up(n: int, m: int) -> int:
    return ((n + m - 1) // m) * m


# ------------------------------------------------------- tensor parallelism
def shard_config(cfg: ModelConfig, tp: int, vocab_rank: Optional[int] = None) -> ModelConfig:
    """Per-rank config of a tensor-parallel Gemma: query / KV heads and the MLP
    width split over ``tp`` ranks (Megatron column split of q/k/v and gate/up,
    row split of o and down), embedding and norms replicated.  The LM head is
    replicated too, unless ``vocab_rank`` names this rank: then a greedy graph
    computes the logits of its vocabulary shard only (rows of the tied
    embedding, read in place) and the ranks agree on the token through two
    max all-reduces (``vocab_split_greedy``).  An addition of this repository;
    the reference runs on one device."""
    if tp == 1:
        return cfg
    if cfg.family == "gpt2":
        raise ValueError("tensor parallelism is provided for the Gemma families")
    if cfg.n_heads % tp or cfg.n_kv_heads % tp or cfg.mlp % tp:
        raise ValueError(f"heads {cfg.n_heads}/{cfg.n_kv_heads} and MLP {cfg.mlp} must divide by tp={tp}")
    if vocab_rank is not None and (cfg.vocab % tp or not 0 <= vocab_rank < tp):
        raise ValueError(f"vocabulary {cfg.vocab} must divide by tp={tp} (rank {vocab_rank})")
    return replace(cfg, n_heads=cfg.n_heads // tp, n_kv_heads=cfg.n_kv_heads // tp, mlp=cfg.mlp // tp, tp=tp,
                   vocab_rank=vocab_rank)


def shard_weights(cfg: ModelConfig, weights: List[np.ndarray], rank: int, tp: int) -> List[np.ndarray]:
    """Rank ``rank``'s slices of the full weights (invar order of weight_specs)."""
    if tp == 1:
        return list(weights)
    out = []
    for (name, shp, _), w in zip(weight_specs(cfg), weights):
        base = name.rsplit("_", 1)[0] if name[-1].isdigit() else name
        if base in ("q_w", "k_w", "v_w", "gate_w", "up_w"):   # column split: rows of [N, K]
            n = w.shape[0] // tp
            out.append(np.ascontiguousarray(w[rank * n:(rank + 1) * n]))
        elif base in ("o_w", "down_w"):                      # row split: columns of [N, K]
            k = w.shape[1] // tp
            out.append(np.ascontiguousarray(w[:, rank * k:(rank + 1) * k]))
        else:
            out.append(w)
    return out


# ------------------------------------------------------------------ invars
def weight_specs(cfg: ModelConfig):
    """(name, shape, kind) per weight invar, in driver order; kind drives the init."""
    d, hd, F = cfg.d_model, cfg.head_dim, cfg.mlp
    q_dim, kv_dim = cfg.n_heads * hd, cfg.n_kv_heads * hd
    specs = []
    if cfg.family == "gpt2":
        specs += [("ln_f_g", (d,), "one"), ("ln_f_b", (d,), "zero"),
                  ("wte", (cfg.vocab, d), "mat"), ("wpe", (cfg.n_positions, d), "mat")]
        for i in range(cfg.layers):
            specs += [(f"ln1_g_{i}", (d,), "one"), (f"ln1_b_{i}", (d,), "zero"),
                      (f"attn_w_{i}", (d, 3 * d), "mat"), (f"attn_b_{i}", (3 * d,), "zero"),
                      (f"proj_w_{i}", (d, d), "mat"), (f"proj_b_{i}", (d,), "zero"),
                      (f"ln2_g_{i}", (d,), "one"), (f"ln2_b_{i}", (d,), "zero"),
                      (f"mlp_fc_w_{i}", (d, F), "mat"), (f"mlp_fc_b_{i}", (F,), "zero"),
                      (f"mlp_proj_w_{i}", (F, d), "mat"), (f"mlp_proj_b_{i}", (d,), "zero")]
        return specs
    # Gemma: (1+w) norms get w ~ N(0, .02); Gemma-3 plain x*w norms get 1 + N(0, .02)
    nk = "plain_norm" if cfg.family == "gemma3" else "gemma_norm"
    specs += [("embed_tokens", (cfg.vocab, d), "mat"), ("final_norm_w", (d,), "gemma_norm")]
    for i in range(cfg.layers):
        specs += [(f"input_ln_w_{i}", (d,), nk), (f"q_w_{i}", (q_dim, d), "mat"),
                  (f"k_w_{i}", (kv_dim, d), "mat"), (f"v_w_{i}", (kv_dim, d), "mat"),
                  (f"o_w_{i}", (d, q_dim), "mat")]
        if cfg.family == "gemma3":
            specs += [(f"q_norm_w_{i}", (hd,), nk), (f"k_norm_w_{i}", (hd,), nk)]
        specs += [(f"post_attn_ln_w_{i}", (d,), nk), (f"pre_mlp_ln_w_{i}", (d,), nk),
                  (f"post_mlp_ln_w_{i}", (d,), nk), (f"gate_w_{i}", (F, d), "mat"),
                  (f"up_w_{i}", (F, d), "mat"), (f"down_w_{i}", (d, F), "mat")]
    return specs


def cache_shape(cfg: ModelConfig, batch: int, max_seq: int):
    return (batch, cfg.n_kv_heads, max_seq, cfg.head_dim)


def graph_invars(cfg: ModelConfig, kind: str, batch: int, prompt_len: int, max_seq: int):
    s = prompt_len if kind == "prefill" else 1
    dt = cfg.dtype
    if cfg.family == "gpt2":
        inv = [("x", ("tensor", (batch, s), "i32")), ("pos_ids", ("tensor", (batch, s), "i32"))]
    else:
        inv = [("x", ("tensor", (batch, s), "i32")), ("pos", ("tensor", (s,), "i32"))]
    inv += [(n, ("tensor", shp, dt)) for n, shp, _ in weight_specs(cfg)]
    cs = cache_shape(cfg, batch, max_seq)
    for i in range(cfg.layers):
        inv += [(f"k_cache_{i}", ("tensor", cs, dt)), (f"v_cache_{i}", ("tensor", cs, dt))]
    return inv


# ------------------------------------------------------------ trace fns
def _gemma_layer_maps(cfg: ModelConfig, weight_args):
    per = 13 if cfg.family == "gemma3" else 11
    maps = []
    for i in range(cfg.layers):
        w = weight_args[i * per:(i + 1) * per]
        if cfg.family == "gemma3":
            m = {"input-ln-w": w[0], "q-w": w[1], "k-w": w[2], "v-w": w[3], "o-w": w[4],
                 "q-norm-w": w[5], "k-norm-w": w[6], "post-attn-ln-w": w[7], "pre-mlp-ln-w": w[8],
                 "post-mlp-ln-w": w[9], "gate-w": w[10], "up-w": w[11], "down-w": w[12],
                 "theta-base": cfg.theta(i), "attn-softcap": cfg.attn_softcap}
        else:
            m = {"input-ln-w": w[0], "q-w": w[1], "k-w": w[2], "v-w": w[3], "o-w": w[4],
                 "post-attn-ln-w": w[5], "pre-mlp-ln-w": w[6], "post-mlp-ln-w": w[7],
                 "gate-w": w[8], "up-w": w[9], "down-w": w[10]}
            if cfg.attn_softcap:
                m["attn-softcap"] = cfg.attn_softcap
        if cfg.is_local(i):
            m["sliding-window"] = cfg.window
        if cfg.tp > 1:
            m["tp"] = cfg.tp
        maps.append(m)
    return maps


def trace_fn(cfg: ModelConfig, kind: str, prompt_len: int, dynamic_prefill: bool = False, greedy: bool = False):
    nw = len(weight_specs(cfg))

    if cfg.family == "gpt2":
        def fn(x, pos_ids, ln_f_g, ln_f_b, wte, wpe, *rest):
            flat, kv = rest[:nw - 4], rest[nw - 4:]
            layers = []
            for i in range(cfg.layers):
                c = flat[i * 12:(i + 1) * 12]
                layers.append({"ln1-g": c[0], "ln1-b": c[1], "c-attn-w": c[2], "c-attn-b": c[3],
                               "c-proj-w": c[4], "c-proj-b": c[5], "ln2-g": c[6], "ln2-b": c[7],
                               "mlp-fc-w": c[8], "mlp-fc-b": c[9], "mlp-proj-w": c[10], "mlp-proj-b": c[11]})
            kv_seq = [[kv[2 * i], kv[2 * i + 1]] for i in range(cfg.layers)]
            if kind == "prefill" and not dynamic_prefill:
                pos = 0
            else:  # cache/mask position = first column of pos_ids, as a [1] tracer
                pos = t.reshape(t.slice(pos_ids, [0, 0], [1, 1], [1, 1]), [1])
            logits, new_kv = full_gpt2_forward(x, pos_ids, ln_f_g, ln_f_b, wte, wpe, layers, kv_seq, pos)
            out = [t.convert(logits, "f32")] if cfg.dtype != "f32" else [logits]
            for k, v in new_kv:
                out += [k, v]
            return out
        return fn

    def fn(x, pos_tr, emb, fnorm, *rest):
        weights, kv = rest[:nw - 2], rest[nw - 2:]
        maps = _gemma_layer_maps(cfg, weights)
        kv_seq = [[kv[2 * i], kv[2 * i + 1]] for i in range(cfg.layers)]
        opts = {"final-logit-softcap": cfg.final_softcap}
        if kind == "prefill" and not dynamic_prefill:
            pos_ids, pos = list(range(prompt_len)), 0
        elif kind == "prefill":
            pos_ids, pos = pos_tr, t.slice(pos_tr, [0], [1], [1])
        else:
            pos_ids, pos = pos_tr, pos_tr
        split = greedy and cfg.vocab_rank is not None
        if split:
            opts["lm-head-rows"] = _vocab_rows(cfg)
        logits, new_kv = full_gemma_forward(x, emb, maps, fnorm, pos_ids, cfg.n_heads, cfg.n_kv_heads,
                                            kv_seq, pos, opts)
        if split:
            out = [vocab_split_greedy(t.convert(logits, "f32"), _vocab_rows(cfg)[0], cfg.tp)]
        else:
            out = [_greedy_token(t.convert(logits, "f32")) if greedy else t.convert(logits, "f32")]
        for k, v in new_kv:
            out += [k, v]
        return out
    return fn


def _greedy_token(logits):
    """In-graph greedy sampling (tensor.clj:519-532 ``argmax`` over the vocabulary,
    as the device-resident decode loop of docs/xla/agent_vram_loop.md:38-80 uses
    it): the next token id [B, S] i32 replaces the f32 logits as the first
    output, so a decode step returns 4 bytes per sequence instead of V * 4.
    Ties take the highest index (the in-graph rule), not argmax-host's lowest."""
    return t.argmax(logits, axis=-1)


def _vocab_rows(cfg: ModelConfig):
    """[first, last) vocabulary rows of this rank's LM-head shard."""
    n = cfg.vocab // cfg.tp
    return cfg.vocab_rank * n, (cfg.vocab_rank + 1) * n


def vocab_split_greedy(logits, first_row: int, tp: int):
    """The greedy token of a vocabulary-sharded LM head: each rank holds the
    logits of rows [first_row, first_row + V / tp).  Its local argmax (highest
    index on ties, tensor.clj:519-532) and local maximum go through two max
    all-reduces: the group's maximum, then the largest global index among the
    ranks that reach it, which is the unsharded argmax's highest-index tie
    rule.  Replaces the replicated LM head's V x d weight read per rank by
    V / tp x d, and the logits never leave their rank."""
    local_max = t.reduce_max(logits, axes=[-1], keep_dims=False)
    local_idx = t.add(t.argmax(logits, axis=-1), first_row)
    top = t.all_reduce(local_max, tp, "max")
    cand = t.select(t.eq(local_max, top), local_idx, -1)
    return t.all_reduce(cand, tp, "max")


def build_graph(cfg: ModelConfig, kind: str, batch: int, prompt_len: int, max_seq: int,
                dynamic_prefill: bool = False, name: Optional[str] = None, greedy: bool = False) -> dict:
    """``greedy=True`` (Gemma families): the first output is the in-graph argmax
    token id [B, S] i32 instead of the f32 logits."""
    inv = graph_invars(cfg, kind, batch, prompt_len, max_seq)
    gname = name or f"{cfg.family}_{kind}" + ("_greedy" if greedy else "")
    if greedy and cfg.family == "gpt2":
        raise ValueError("in-graph greedy sampling is provided for the Gemma families")
    return t.trace_graph(gname, inv, trace_fn(cfg, kind, prompt_len, dynamic_prefill, greedy))


# ------------------------------------------------------- synthetic inputs
def _to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, returned as uint16 bit patterns."""
    u = np.asarray(a, dtype=np.float32, order="C").view(np.uint32)
    rounded = u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))
    out = (rounded >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def make_weights(cfg: ModelConfig, seed: int = 0) -> List[np.ndarray]:
    """Random-init weights in invar order from PCG64(seed).

    Matrices / embeddings ~ N(0, 0.02); (1+w) norms w ~ N(0, 0.02); plain norms
    1 + N(0, 0.02); GPT-2 LN gamma = 1, beta / biases = 0.  bf16 configs return
    uint16 bf16 bit patterns, f32 configs float32 arrays.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    for name, shp, kind in weight_specs(cfg):
        if kind == "mat":
            a = (rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02))
        elif kind == "gemma_norm":
            a = rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        elif kind == "plain_norm":
            a = np.float32(1.0) + rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        elif kind == "one":
            a = np.ones(shp, np.float32)
        else:
            a = np.zeros(shp, np.float32)
        out.append(_to_bf16_bits(a) if cfg.dtype == "bf16" else a.astype(np.float32))
    return out


def device_weights(cfg: ModelConfig, seed: int, device: str = "cuda:0") -> List[np.ndarray]:
    """Seeded random-init weights in invar order, drawn on the GPU with torch
    (a few seconds for the largest configs, where a host generator takes
    minutes), returned as host arrays ready for BufferFromHostBuffer: bf16 bit
    patterns (uint16) for bf16 configs, float32 otherwise.  Same distributions
    as ``make_weights``."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = []
    for name, shp, kind in weight_specs(cfg):
        if kind in ("mat", "gemma_norm"):
            w = torch.randn(shp, generator=g, device=device, dtype=torch.float32).mul_(0.02)
        elif kind == "plain_norm":
            w = torch.randn(shp, generator=g, device=device, dtype=torch.float32).mul_(0.02).add_(1.0)
        elif kind == "one":
            w = torch.ones(shp, device=device)
        else:
            w = torch.zeros(shp, device=device)
        if cfg.dtype == "bf16":
            out.append(w.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16))
        else:
            out.append(w.cpu().numpy())
        del w
    return out


def make_prompt(cfg: ModelConfig, batch: int, prompt_len: int, seed: int = 1) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(0, cfg.vocab, size=(batch, prompt_len), dtype=np.int64).astype(np.int32)


def zero_cache(cfg: ModelConfig, batch: int, max_seq: int) -> np.ndarray:
    shp = cache_shape(cfg, batch, max_seq)
    return np.zeros(shp, np.uint16 if cfg.dtype == "bf16" else np.float32)


def pos_inputs(cfg: ModelConfig, kind: str, batch: int, start: int, length: int) -> np.ndarray:
    """The ``pos`` / ``pos_ids`` invar value for a prefill (start=0) or decode step."""
    p = np.arange(start, start + length, dtype=np.int32)
    if cfg.family == "gpt2":
        return np.broadcast_to(p, (batch, length)).copy()
    return p


def argmax_host(logits_row: np.ndarray) -> int:
    """scripts/gemma4_inference.clj:399-411 - first (lowest) index of the maximum."""
    return int(np.argmax(logits_row))
