"""GPT-2 and Gemma-1/2/3 forward functions traced into SSA graphs.

Host-side mirror of ``src/clj_xla/models/gpt2.clj:22-75`` and
``src/clj_xla/models/gemma.clj:8-23,122-280``.  One addition, marked where it
happens: a layer map may carry ``"sliding-window"``, which is forwarded into
``gqa_causal_attention``'s opts (the reference's ``gqa-causal-attention``
accepts it at attention.clj:355 but ``gemma-attention`` drops it at
gemma.clj:180).  Without that key the traced graph is the reference's.
"""
from __future__ import annotations

import math

from . import tensor as t
from .nn import (apply_rope, gelu, gemma_rms_norm, gqa_causal_attention, layer_norm,
                 causal_self_attention, rms_norm, rms_norm_split, linear as attn_linear)


# ------------------------------------------------------------------ gpt2.clj
def _gpt2_embed(x, pos_ids, wte, wpe):
    """gpt2.clj:22-25."""
    tok = t.gather(wte, x)
    pos = t.gather(wpe, pos_ids)
    return t.add(tok, pos)


def gpt2_mlp(x, fc_w, fc_b, proj_w, proj_b):
    """gpt2.clj:27-31."""
    h = gelu(attn_linear(x, fc_w, fc_b))
    return attn_linear(h, proj_w, proj_b)


def gpt2_block(x, w, num_heads, past_kv=None, pos=None):
    """gpt2.clj:33-50."""
    xn1 = layer_norm(x, w["ln1-g"], w["ln1-b"])
    if past_kv is not None:
        res = causal_self_attention(xn1, w["c-attn-w"], w["c-attn-b"], w["c-proj-w"], w["c-proj-b"],
                                    num_heads, past_kv, pos)
    else:
        res = causal_self_attention(xn1, w["c-attn-w"], w["c-attn-b"], w["c-proj-w"], w["c-proj-b"], num_heads)
    attn_out, updated = (res[0], res[1]) if isinstance(res, list) else (res, None)
    r1 = t.add(x, attn_out)
    xn2 = layer_norm(r1, w["ln2-g"], w["ln2-b"])
    mlp = gpt2_mlp(xn2, w["mlp-fc-w"], w["mlp-fc-b"], w["mlp-proj-w"], w["mlp-proj-b"])
    out = t.add(r1, mlp)
    return [out, updated] if past_kv is not None else out


def full_gpt2_forward(x, pos_ids, ln_f_g, ln_f_b, wte, wpe, layers, kv_caches=None, pos=None):
    """gpt2.clj:52-75 (12 heads hard-coded as in the reference)."""
    h = _gpt2_embed(x, pos_ids, wte, wpe)
    new_kv = None
    if kv_caches is not None:
        new_kv = []
        for lw, kv in zip(layers, kv_caches):
            h, nk = gpt2_block(h, lw, 12, kv, pos)
            new_kv.append(nk)
    else:
        for lw in layers:
            h = gpt2_block(h, lw, 12)
    normed = layer_norm(h, ln_f_g, ln_f_b)
    logits = attn_linear(normed, t.transpose(wte, [1, 0]), None)
    return [logits, new_kv] if kv_caches is not None else logits


# ----------------------------------------------------------------- gemma.clj
def gemma_linear(x, w, b=None):
    """gemma.clj:8-23 - contract the weight dim that matches x's last dim."""
    tx = t.emit_constant(x, None)
    tw = t.emit_constant(w, None)
    xs, ws = tx.type[1], tw.type[1]
    xr, wr = len(xs), len(ws)
    contract_rhs = 0 if ws[0] == xs[-1] else wr - 1
    if xr == 2 and wr == 2 and ws[0] == xs[-1]:
        out = t.matmul(tx, tw)
    else:
        out = t.dot_general(tx, tw, {"contracting_dims": {"lhs": [xr - 1], "rhs": [contract_rhs]}})
    return t.add(out, b) if b is not None else out


def gemma_embed_lookup(x, embed, hidden_dim):
    """gemma.clj:122-126 - gather then scale by sqrt(d)."""
    raw = t.gather(embed, x)
    h_dim = hidden_dim or embed.type[1][1]
    return t.mul(raw, math.sqrt(float(h_dim)))


def gemma_mlp(x, gate_w, up_w, down_w):
    """gemma.clj:128-137 - GeGLU."""
    gate_t = t.transpose(gate_w, [1, 0])
    up_t = t.transpose(up_w, [1, 0])
    down_t = t.transpose(down_w, [1, 0])
    gate_out = gelu(gemma_linear(x, gate_t, None))
    up_out = gemma_linear(x, up_t, None)
    hidden = t.mul(gate_out, up_out)
    return gemma_linear(hidden, down_t, None)


def gemma_attention(x, q_w, k_w, v_w, o_w, num_heads, _num_kv_heads, pos_ids, past_kv=None, pos=None, opts=None):
    """gemma.clj:139-189 (shared-KV branch of Gemma-4 omitted)."""
    opts = opts or {}
    q_norm_w = opts.get("q-norm-w")
    k_norm_w = opts.get("k-norm-w")
    theta = opts.get("theta-base") or 10000.0
    softcap = opts.get("attn-softcap")
    rotary_dim = opts.get("rotary-dim")
    rope_prop = opts.get("rope-proportion") or 1.0
    norm_fn = opts.get("norm-fn") or (rms_norm if q_norm_w is not None else gemma_rms_norm)
    q = gemma_linear(x, t.transpose(q_w, [1, 0]), None)
    qs = q.type[1]
    batch = qs[0] if len(qs) == 3 else 1
    seq_len = qs[1] if len(qs) == 3 else 1
    q_proj = qs[-1]
    h_dim = opts.get("head-dim") or q_proj // num_heads
    q4 = t.transpose(t.reshape(q, [batch, seq_len, num_heads, h_dim]), [0, 2, 1, 3])
    q_normed = norm_fn(q4, q_norm_w, 1e-6) if q_norm_w is not None else q4
    k_w_t = t.transpose(k_w, [1, 0])
    v_w_t = t.transpose(v_w, [1, 0])
    k = gemma_linear(x, k_w_t, None)
    v_raw = gemma_linear(x, v_w_t, None)
    tp = opts.get("tp", 1)
    if q_norm_w is not None:
        v = rms_norm(v_raw, None, 1e-6) if tp == 1 else rms_norm_split(v_raw, 1e-6, tp)
    else:
        v = v_raw
    kv_dim = k.type[1][-1]
    l_nkv = kv_dim // h_dim
    k4 = t.transpose(t.reshape(k, [batch, seq_len, l_nkv, h_dim]), [0, 2, 1, 3])
    k_normed = norm_fn(k4, k_norm_w, 1e-6) if k_norm_w is not None else k4
    _, k_rope = apply_rope(q_normed, k_normed, pos_ids, h_dim, theta, rotary_dim, None, rope_prop)
    k3 = t.reshape(t.transpose(k_rope, [0, 2, 1, 3]), [batch, seq_len, kv_dim])
    q_rope, _ = apply_rope(q_normed, q_normed, pos_ids, h_dim, theta, rotary_dim, None, rope_prop)
    q3 = t.reshape(t.transpose(q_rope, [0, 2, 1, 3]), [batch, seq_len, q_proj])
    scale = opts.get("scale", 1.0 if q_norm_w is not None else 1.0 / math.sqrt(float(h_dim)))
    attn_opts = {"scale": scale}
    if opts.get("sliding-window"):  # added key, see module docstring
        attn_opts["sliding-window"] = opts["sliding-window"]
    l_nkv = k3.type[1][-1] // h_dim
    if past_kv is not None:
        res = gqa_causal_attention(q3, k3, v, o_w, num_heads, l_nkv, softcap, past_kv, pos, attn_opts)
        return [res[0], res[1], [k3, v]]
    res = gqa_causal_attention(q3, k3, v, o_w, num_heads, l_nkv, softcap, None, None, attn_opts)
    return [res, None, [k3, v]]


def gemma_block(x, w, num_heads, num_kv_heads, pos_ids, past_kv=None, pos=None):
    """gemma.clj:191-244 (Gemma-4 PLE / layer-scalar branches omitted)."""
    q_norm_w = w.get("q-norm-w")
    norm_fn = w.get("norm-fn") or (rms_norm if q_norm_w is not None else gemma_rms_norm)
    xn1 = norm_fn(x, w["input-ln-w"], 1e-6)
    attn_opts = {"q-norm-w": q_norm_w, "k-norm-w": w.get("k-norm-w"),
                 "theta-base": w.get("theta-base", 10000.0), "attn-softcap": w.get("attn-softcap"),
                 "rotary-dim": w.get("rotary-dim"), "head-dim": w.get("head-dim"),
                 "rope-proportion": w.get("rope-proportion", 1.0), "norm-fn": norm_fn,
                 "sliding-window": w.get("sliding-window"), "tp": w.get("tp", 1)}
    attn_raw, updated, _ = gemma_attention(xn1, w["q-w"], w["k-w"], w["v-w"], w["o-w"], num_heads, num_kv_heads,
                                           pos_ids, past_kv, pos, attn_opts)
    tp = w.get("tp", 1)
    if tp > 1:  # tensor parallel: the o-projection of the local heads is a partial sum
        attn_raw = t.all_reduce(attn_raw, tp)
    pa = w.get("post-attn-ln-w")
    attn_normed = norm_fn(attn_raw, pa, 1e-6) if pa is not None else attn_raw
    attn_out = t.add(attn_normed, x)
    pm = w.get("pre-mlp-ln-w")
    xn2 = norm_fn(attn_out, pm, 1e-6) if pm is not None else attn_out
    mlp_raw = gemma_mlp(xn2, w["gate-w"], w["up-w"], w["down-w"])
    if tp > 1:  # the down-projection of the local MLP slice is a partial sum
        mlp_raw = t.all_reduce(mlp_raw, tp)
    po = w.get("post-mlp-ln-w")
    mlp_normed = norm_fn(mlp_raw, po, 1e-6) if po is not None else mlp_raw
    out = t.add(mlp_normed, attn_out)
    return [out, updated] if past_kv is not None else out


def full_gemma_forward(x, embed, layers, final_norm_w, pos_ids, num_heads, num_kv_heads,
                       kv_caches=None, pos=None, opts=None):
    """gemma.clj:246-280 - final norm is always the (1+w) Gemma RMSNorm."""
    opts = opts or {}
    hidden = embed.type[1][1]
    h = gemma_embed_lookup(x, embed, hidden)
    new_kv = None
    if kv_caches is not None:
        new_kv = []
        for lw, kv in zip(layers, kv_caches):
            h, nk = gemma_block(h, lw, num_heads, num_kv_heads, pos_ids, kv, pos)
            new_kv.append(nk)
    else:
        for lw in layers:
            h = gemma_block(h, lw, num_heads, num_kv_heads, pos_ids)
    normed = gemma_rms_norm(h, final_norm_w, 1e-6)
    rows = opts.get("lm-head-rows")
    if rows is not None:
        # vocabulary-sharded LM head (tensor parallelism, an addition of this
        # repository): this rank's rows of the tied embedding, a view in place
        embed = t.slice(embed, [rows[0], 0], [rows[1], hidden], [1, 1])
    embed_t = t.transpose(embed, [1, 0])
    raw = gemma_linear(normed, embed_t, None)
    fs = opts.get("final-logit-softcap", 30.0)
    if isinstance(fs, (int, float)) and fs > 0:
        logits = t.mul(fs, t.tanh(t.div(raw, fs)))
    else:
        logits = raw
    return [logits, new_kv] if kv_caches is not None else logits
