"""Decoder building blocks traced into SSA equations.

Host-side mirror of ``src/clj_xla/nn/attention.clj`` (linear, RoPE, KV-cache
update, causal mask, MHA, GQA), ``src/clj_xla/nn/norm.clj`` (LayerNorm,
RMSNorm, Gemma RMSNorm) and ``src/clj_xla/nn/activations.clj:7-11`` (GELU-tanh).
The op sequence, constants and tracer-side dtypes follow the reference so that
the printed graph is the one the reference host would send.
"""
from __future__ import annotations

import math

from . import tensor as t
from .tensor import Tracer, tracer_p


# ----------------------------------------------------------------- norm.clj
def layer_norm(x, gamma, beta, eps=1e-5):
    """norm.clj:6-15."""
    mu = t.reduce_mean(x, axes=[-1], keep_dims=True)
    diff = t.sub(x, mu)
    var = t.reduce_mean(t.pow(diff, 2.0), axes=[-1], keep_dims=True)
    x_hat = t.div(diff, t.sqrt(t.add(var, eps)))
    return t.add(t.mul(x_hat, gamma), beta)


def rms_norm(x, weight, eps=1e-6):
    """norm.clj:17-26 - ``x / sqrt(mean(x^2) + eps) * w`` (no weight: plain)."""
    ms = t.reduce_mean(t.pow(x, 2.0), axes=[-1], keep_dims=True)
    x_hat = t.div(x, t.sqrt(t.add(ms, eps)))
    if weight is not None:
        return t.mul(x_hat, weight)
    return x_hat


def rms_norm_split(x, eps, tp):
    """``rms_norm(x, None, eps)`` when the last dimension of ``x`` is split over
    ``tp`` tensor-parallel ranks: the local sums of squares are all-reduced so
    every rank divides by the root mean square of the whole, unsplit row (the
    Gemma-3 value projection is normalised across all heads, gemma.clj:166-167).
    An addition of this repository for tensor parallelism."""
    tx = t.emit_constant(x, None)
    full = tx.type[1][-1] * tp
    ss = t.all_reduce(t.reduce_sum(t.pow(tx, 2.0), axes=[-1], keep_dims=True), tp)
    ms = t.div(ss, float(full))
    return t.div(tx, t.sqrt(t.add(ms, eps)))


def gemma_rms_norm(x, weight, eps=1e-6):
    """norm.clj:28-35 - ``... * (1 + w)``."""
    ms = t.reduce_mean(t.pow(x, 2.0), axes=[-1], keep_dims=True)
    x_hat = t.div(x, t.sqrt(t.add(ms, eps)))
    return t.mul(x_hat, t.add(1.0, weight))


# ---------------------------------------------------------- activations.clj
def gelu(x):
    """activations.clj:7-11 - tanh approximation, ``(* 0.5 x (+ 1 ...))``."""
    c_sqrt = 0.7978845608
    # (* 0.5 x Y): Clojure evaluates Y before the variadic multiply folds left
    return t.mul(0.5, x, t.add(1.0, t.tanh(t.mul(c_sqrt, t.add(x, t.mul(0.044715, t.pow(x, 3.0)))))))


# ------------------------------------------------------------ attention.clj
def linear(x, w, b=None):
    """attention.clj:6-10 - ``x @ w (+ b)``."""
    h = t.matmul(x, w)
    return t.add(h, b) if b is not None else h


def _extract_pos_int(pos) -> int:
    """attention.clj:12-17."""
    if pos is None:
        return 0
    if isinstance(pos, (int, float)) and not isinstance(pos, bool):
        return int(pos)
    if isinstance(pos, (list, tuple)):
        return int(pos[0]) if len(pos) else 0
    return 0


def _rope_freq_tensors(seq_len, head_dim, theta_base, pos_offset, full_dim=None, rope_proportion=1.0):
    """attention.clj:19-61 - dynamic (tracer pos) or static constant cos/sin tables."""
    f_dim = full_dim or head_dim
    t_base = theta_base or 10000.0
    rope_prop = float(rope_proportion if rope_proportion is not None else 1.0)
    half = head_dim // 2
    angles_n = int(rope_prop * half)
    freqs = [math.pow(t_base, (-2.0 * i) / float(f_dim)) if i < angles_n else 0.0 for i in range(half)]
    if tracer_p(pos_offset):
        freqs_c = t.emit_constant([[[[*freqs]]]], ("tensor", (1, 1, 1, half), "f32"))
        pos_f32 = t.convert(pos_offset, "f32")
        ps = pos_f32.type[1]
        if len(ps) == 2:
            s_len = ps[1]
        elif len(ps) == 0:
            s_len = 1
        else:
            s_len = ps[0] or 1
        pos4 = t.reshape(pos_f32, [1, 1, s_len, 1])
        ang = t.mul(pos4, freqs_c)
        c_h = t.cos(ang)
        s_h = t.sin(ang)
        return t.concatenate([c_h, c_h], 3), t.concatenate([s_h, s_h], 3)
    p_off = _extract_pos_int(pos_offset)
    cos_rows, sin_rows = [], []
    for idx in range(seq_len):
        p = float(p_off + idx)
        ch = [math.cos(p * freqs[i]) for i in range(half)]
        sh = [math.sin(p * freqs[i]) for i in range(half)]
        cos_rows.append(ch + ch)
        sin_rows.append(sh + sh)
    return (t.emit_constant([[cos_rows]], ("tensor", (1, 1, seq_len, head_dim), "f32")),
            t.emit_constant([[sin_rows]], ("tensor", (1, 1, seq_len, head_dim), "f32")))


def _apply_rope_single(x, pos_ids, head_dim, theta_base, rotary_dim=None, full_dim=None, rope_proportion=1.0):
    """attention.clj:63-108."""
    _, shape, dtype = x.type
    t_base = theta_base or 10000.0
    if len(shape) == 3:
        batch, seq_len, q_dim = shape
        h_dim = head_dim or 64
        n_heads = q_dim // h_dim
        x4 = t.transpose(t.reshape(x, [batch, seq_len, n_heads, h_dim]), [0, 2, 1, 3])
        r4 = _apply_rope_single(x4, pos_ids, h_dim, t_base, rotary_dim, full_dim or h_dim, rope_proportion)
        return t.reshape(t.transpose(r4, [0, 2, 1, 3]), [batch, seq_len, q_dim])
    batch, num_heads, seq_len, h_dim = shape
    f_dim = full_dim or h_dim
    rope_prop = float(rope_proportion if rope_proportion is not None else 1.0)
    r_dim = int(rotary_dim if rotary_dim is not None else float(f_dim) * rope_prop)
    if r_dim < h_dim:
        x_rope = t.slice(x, [0, 0, 0, 0], [batch, num_heads, seq_len, r_dim], [1, 1, 1, 1])
        x_pass = t.slice(x, [0, 0, 0, r_dim], [batch, num_heads, seq_len, h_dim], [1, 1, 1, 1])
        half = r_dim // 2
        x1 = t.slice(x_rope, [0, 0, 0, 0], [batch, num_heads, seq_len, half], [1, 1, 1, 1])
        x2 = t.slice(x_rope, [0, 0, 0, half], [batch, num_heads, seq_len, r_dim], [1, 1, 1, 1])
        x_rot = t.concatenate([t.sub(x2), x1], -1)
        cos_t, sin_t = _rope_freq_tensors(seq_len, r_dim, t_base, pos_ids, r_dim, 1.0)
        res_rope = t.add(t.mul(x_rope, cos_t), t.mul(x_rot, sin_t))
        return t.concatenate([t.convert(res_rope, dtype), t.convert(x_pass, dtype)], -1)
    half = f_dim // 2
    x1 = t.slice(x, [0, 0, 0, 0], [batch, num_heads, seq_len, half], [1, 1, 1, 1])
    x2 = t.slice(x, [0, 0, 0, half], [batch, num_heads, seq_len, f_dim], [1, 1, 1, 1])
    x_rot = t.concatenate([t.sub(x2), x1], -1)
    cos_t, sin_t = _rope_freq_tensors(seq_len, f_dim, t_base, pos_ids, f_dim, 1.0)
    res = t.add(t.mul(x, cos_t), t.mul(x_rot, sin_t))
    return res if dtype == "f32" else t.convert(res, dtype)


def apply_rope(x, y, z, head_dim=None, theta_base=10000.0, rotary_dim=None, full_dim=None, rope_proportion=1.0):
    """attention.clj:110-133 (the 8-arity form; ``y`` may be nil)."""
    if y is not None:
        return [apply_rope(x, None, z, head_dim, theta_base, rotary_dim, full_dim, rope_proportion),
                apply_rope(y, None, z, head_dim, theta_base, rotary_dim, full_dim, rope_proportion)]
    shape = x.type[1]
    h_dim = head_dim or (shape[3] if len(shape) == 4 else 64)
    return _apply_rope_single(x, z, h_dim, theta_base, rotary_dim, full_dim or h_dim, rope_proportion)


def _update_single_cache(cache, new_val, pos):
    """attention.clj:135-168 - DUS at the seq dim; static pos also slices the active prefix."""
    if cache is None:
        return new_val, new_val
    _, shape, cache_dtype = cache.type
    rank = len(shape)
    seq_dim = rank - 2
    max_len = shape[seq_dim]
    _, new_shape, nv_dtype = new_val.type
    ln = new_shape[seq_dim]
    pos_val = pos if tracer_p(pos) else _extract_pos_int(pos)
    starts = [0] * rank
    starts[seq_dim] = pos_val
    nv_typed = new_val if cache_dtype == nv_dtype else t.convert(new_val, cache_dtype)
    should_slice = ln > 0 and max_len > 0 and ln > max_len
    if should_slice:
        sliced = t.slice(nv_typed, [0, 0, ln - max_len, 0], list(new_shape), [1, 1, 1, 1])
        eff = [0] * rank
    else:
        sliced = nv_typed
        eff = starts
    updated = t.dynamic_update_slice(cache, sliced, eff)
    if tracer_p(pos):
        active = updated
    else:
        end_pos = min(pos_val + ln, max_len)
        lim = list(shape)
        lim[seq_dim] = end_pos
        active = updated if end_pos == max_len else t.slice(updated, [0] * rank, lim, [1] * rank)
    return updated, active


def update_kv_cache(past_kv, new_k, new_v, pos):
    """attention.clj:170-184."""
    k_cache, v_cache = past_kv
    uk, ak = _update_single_cache(k_cache, new_k, pos)
    uv, av = _update_single_cache(v_cache, new_v, pos)
    return [uk, uv], [ak, av]


def generate_causal_mask(q_len, kv_len, pos, sliding_window=None):
    """attention.clj:186-225 - additive -10000 mask (iota/compare/select if pos is a tracer)."""
    if tracer_p(pos):
        i_iota = t.convert(t.iota(q_len, "i32"), "f32")
        j_iota = t.convert(t.iota(kv_len, "i32"), "f32")
        i_c = t.reshape(i_iota, [1, 1, q_len, 1])
        j_c = t.reshape(j_iota, [1, 1, 1, kv_len])
        if tuple(pos.type[1]) in ((1,), ()):
            p_c = t.reshape(t.convert(pos, "f32"), [1, 1, 1, 1])
        else:
            p_c = t.emit_constant(0.0, ("tensor", (1, 1, 1, 1), "f32"))
        eff_i = t.add(i_c, p_c)
        diff = t.sub(j_c, eff_i)
        zero4 = t.broadcast_in_dim(t.reshape(t.emit_constant([0.0], ("tensor", (1,), "f32")), [1, 1, 1, 1]),
                                   [1, 1, q_len, kv_len], [0, 1, 2, 3])
        mask_val = t.broadcast_in_dim(t.reshape(t.emit_constant([-10000.0], ("tensor", (1,), "f32")), [1, 1, 1, 1]),
                                      [1, 1, q_len, kv_len], [0, 1, 2, 3])
        gt_zero = t.compare_t(diff, zero4, "GT")
        masked_gt = t.select(gt_zero, mask_val, zero4)
        if isinstance(sliding_window, (int, float)) and sliding_window > 0:
            sw = float(-float(sliding_window))
            sw4 = t.broadcast_in_dim(t.reshape(t.emit_constant([sw], ("tensor", (1,), "f32")), [1, 1, 1, 1]),
                                     [1, 1, q_len, kv_len], [0, 1, 2, 3])
            lt_sw = t.compare_t(diff, sw4, "LT")
            return t.select(lt_sw, mask_val, masked_gt)
        return masked_gt
    p = _extract_pos_int(pos)
    rows = []
    for i in range(q_len):
        pi = p + i
        row = []
        for j in range(kv_len):
            too_far = isinstance(sliding_window, (int, float)) and sliding_window > 0 and j < pi - sliding_window
            row.append(-10000.0 if (j > pi or too_far) else 0.0)
        rows.append(row)
    return t.emit_constant([[rows]], ("tensor", (1, 1, q_len, kv_len), "f32"))


def causal_self_attention(x, c_attn_w, c_attn_b, c_proj_w, c_proj_b, num_heads, past_kv=None, pos=None):
    """attention.clj:227-285 - GPT-2 MHA (fused qkv projection, scale 1/sqrt(hd))."""
    batch, seq_len, _ = x.type[1]
    num_heads = num_heads or 12
    qkv = linear(x, c_attn_w, c_attn_b)
    qkv_dim = qkv.type[1][2]
    embed = qkv_dim // 3
    hd = embed // num_heads
    q = t.slice(qkv, [0, 0, 0], [batch, seq_len, embed], [1, 1, 1])
    k = t.slice(qkv, [0, 0, embed], [batch, seq_len, 2 * embed], [1, 1, 1])
    v = t.slice(qkv, [0, 0, 2 * embed], [batch, seq_len, qkv_dim], [1, 1, 1])
    qh = t.transpose(t.reshape(q, [batch, seq_len, num_heads, hd]), [0, 2, 1, 3])
    kh = t.transpose(t.reshape(k, [batch, seq_len, num_heads, hd]), [0, 2, 1, 3])
    vh = t.transpose(t.reshape(v, [batch, seq_len, num_heads, hd]), [0, 2, 1, 3])
    if past_kv is not None:
        updated, (ka, va) = update_kv_cache(past_kv, kh, vh, pos if pos is not None else 0)
    else:
        updated, (ka, va) = None, (kh, vh)
    kv_len = ka.type[1][2]
    scale = 1.0 / math.sqrt(float(hd))
    raw = t.dot_general(qh, ka, {"batch_dims": {"lhs": [0, 1], "rhs": [0, 1]},
                                  "contracting_dims": {"lhs": [3], "rhs": [3]}})
    scaled = t.mul(raw, scale)
    mask = generate_causal_mask(seq_len, kv_len, pos if pos is not None else 0)
    masked = t.add(scaled, mask)
    mx = t.reduce_max(masked, axes=[-1], keep_dims=True)
    ex = t.exp(t.sub(masked, mx))
    sm = t.reduce_sum(ex, axes=[-1], keep_dims=True)
    probs = t.div(ex, sm)
    ctx = t.dot_general(probs, va, {"batch_dims": {"lhs": [0, 1], "rhs": [0, 1]},
                                    "contracting_dims": {"lhs": [3], "rhs": [2]}})
    merged = t.reshape(t.transpose(ctx, [0, 2, 1, 3]), [batch, seq_len, embed])
    out = linear(merged, c_proj_w, c_proj_b)
    if past_kv is not None:
        return [out, updated]
    return out


def gqa_causal_attention(q, k, v, o_w, num_heads, num_kv_heads, attn_softcap=None,
                         past_kv=None, pos=None, opts=None):
    """attention.clj:287-375 - GQA via broadcast+reshape of K/V, optional softcap."""
    opts = opts or {}
    q_shape = q.type[1]
    k_shape = k.type[1]
    q4 = len(q_shape) == 4
    k4 = len(k_shape) == 4
    batch = q_shape[0]
    q_len = q_shape[2] if q4 else q_shape[1]
    q_dim = q_shape[1] * q_shape[3] if q4 else q_shape[2]
    num_heads = num_heads or 8
    num_kv_heads = num_kv_heads or 4
    hd = q_dim // num_heads
    k_dim = k_shape[1] * k_shape[3] if k4 else k_shape[2]
    nkv = k_dim // hd if hd > 0 else num_kv_heads
    k_4d = k if k4 else t.transpose(t.reshape(k, [batch, q_len, nkv, hd]), [0, 2, 1, 3])
    v_4d = v if k4 else t.transpose(t.reshape(v, [batch, q_len, nkv, hd]), [0, 2, 1, 3])
    if past_kv is not None:
        updated, (ka, va) = update_kv_cache(past_kv, k_4d, v_4d, pos if pos is not None else 0)
    else:
        updated, (ka, va) = None, (k_4d, v_4d)
    kv_len = ka.type[1][2]
    group = num_heads // nkv
    scale = opts.get("scale", 1.0 / math.sqrt(float(hd)))
    qh = q if q4 else t.transpose(t.reshape(q, [batch, q_len, num_heads, hd]), [0, 2, 1, 3])
    if group == 1:
        kh, vh = ka, va
    else:
        k_rep = t.broadcast_in_dim(ka, [batch, num_kv_heads, group, kv_len, hd], [0, 1, 3, 4])
        v_rep = t.broadcast_in_dim(va, [batch, num_kv_heads, group, kv_len, hd], [0, 1, 3, 4])
        kh = t.reshape(k_rep, [batch, num_heads, kv_len, hd])
        vh = t.reshape(v_rep, [batch, num_heads, kv_len, hd])
    raw = t.dot_general(qh, kh, {"batch_dims": {"lhs": [0, 1], "rhs": [0, 1]},
                                  "contracting_dims": {"lhs": [3], "rhs": [3]}})
    scaled = t.mul(raw, scale)
    if isinstance(attn_softcap, (int, float)) and attn_softcap > 0:
        capped = t.mul(attn_softcap, t.tanh(t.div(scaled, attn_softcap)))
    else:
        capped = scaled
    mask = generate_causal_mask(q_len, kv_len, pos if pos is not None else 0, opts.get("sliding-window"))
    masked = t.add(capped, mask)
    mx = t.reduce_max(masked, axes=[-1], keep_dims=True)
    ex = t.exp(t.sub(masked, mx))
    sm = t.reduce_sum(ex, axes=[-1], keep_dims=True)
    probs = t.div(ex, sm)
    ctx = t.dot_general(probs, vh, {"batch_dims": {"lhs": [0, 1], "rhs": [0, 1]},
                                    "contracting_dims": {"lhs": [3], "rhs": [2]}})
    merged = t.reshape(t.transpose(ctx, [0, 2, 1, 3]), [batch, q_len, q_dim])
    o_w_t = t.transpose(o_w, [1, 0])
    out = linear(merged, o_w_t, None)
    if past_kv is not None:
        return [out, updated]
    return out
