"""Pins the CPU oracle (oracle/interp.py) before it is trusted as the checker.

* the reference's one numeric known-answer test: rocm_e2e_test.clj:38-51,
  ``y = 2.5 * x`` for x = 0..15 within atol = rtol = 1e-4 (parity.clj:36-49);
* StableHLO semantics the model graphs rely on: bf16 rounding, reduce init,
  clamped gather / dynamic_update_slice indices, the in-graph argmax tie rule
  (tensor.clj:519-532: highest index wins);
* static and dynamic (tracer-position) graphs of the same model agree.
"""
import dataclasses

import numpy as np
import pytest

from cljxla_b200.host import drivers as d
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200.host import tensor as t
from oracle import interp


def approx_equal(a, b, atol=1e-4, rtol=1e-4):
    """parity.clj:36-49 ``approx-equal?``."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return a.shape == b.shape and bool(np.all(np.abs(a - b) <= atol + rtol * np.abs(b)))


def test_reference_known_answer_2p5x():
    g = {"name": "parity_test_graph", "invars": [("x", ("tensor", (1, 16), "f32"))], "outvars": ["y"],
         "eqns": [{"op": "stablehlo/constant", "value": 2.5, "outvars": ["c0"]},
                  {"op": "stablehlo/multiply", "invars": ["x", "c0"], "outvars": ["y"]}]}
    x = np.arange(16, dtype=np.float32).reshape(1, 16)
    (y,) = interp.run_mlir(shlo.graph_to_mlir_text(g), [x])
    assert approx_equal(y, [v * 2.5 for v in range(16)])


def test_bf16_rounding_is_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.01171875, 1.0078125, -3.14159, 65504.0], np.float32)
    r = interp.round_bf16(vals)
    assert r[1] == 1.0            # exact tie rounds to even
    assert r[2] == 1.015625       # tie rounds up to even
    assert r[3] == 1.0078125      # representable
    bits = interp.f32_to_bf16_bits(vals)
    assert np.array_equal(interp.bf16_bits_to_f32(bits), r)


def test_reduce_max_init_and_argmax_highest_index_on_ties():
    g = t.trace_graph("am", [("x", ("tensor", (1, 6), "f32"))], lambda x: t.argmax(x))
    txt = shlo.graph_to_mlir_text(g)
    (r,) = interp.run_mlir(txt, [np.array([[1, 5, 2, 5, 0, 3]], np.float32)])
    assert int(np.asarray(r).ravel()[0]) == 3
    assert d.argmax_host(np.array([1, 5, 2, 5, 0, 3], np.float32)) == 1


def test_gather_and_dus_clamp_indices():
    emb = np.arange(12, dtype=np.float32).reshape(4, 3)

    def f(e, i):
        return t.gather(e, i)
    g = t.trace_graph("gth", [("e", ("tensor", (4, 3), "f32")), ("i", ("tensor", (1, 3), "i32"))], f)
    (r,) = interp.run_mlir(shlo.graph_to_mlir_text(g), [emb, np.array([[0, 3, 9]], np.int32)])
    assert np.array_equal(r[0], emb[[0, 3, 3]])

    def h(c, u, p):
        return t.dynamic_update_slice(c, u, [0, p])
    g2 = t.trace_graph("dus", [("c", ("tensor", (2, 5), "f32")), ("u", ("tensor", (2, 2), "f32")),
                               ("p", ("tensor", (1,), "i32"))], h)
    c = np.zeros((2, 5), np.float32)
    u = np.ones((2, 2), np.float32)
    (r2,) = interp.run_mlir(shlo.graph_to_mlir_text(g2), [c, u, np.array([4], np.int32)])
    assert np.array_equal(r2[:, 3:], np.ones((2, 2)))   # start clamped to 5-2 = 3


TINY_G3 = dataclasses.replace(d.GEMMA3_4B, vocab=512, d_model=256, layers=2, n_heads=4, n_kv_heads=2,
                              head_dim=64, mlp=512, window=16)


def test_static_and_dynamic_prefill_agree():
    B, S, T = 1, 8, 32
    w = d.make_weights(TINY_G3)
    x = d.make_prompt(TINY_G3, B, S)
    pos = d.pos_inputs(TINY_G3, "prefill", B, 0, S)
    kv = [d.zero_cache(TINY_G3, B, T) for _ in range(2 * TINY_G3.layers)]
    outs = []
    for dyn in (False, True):
        g = d.build_graph(TINY_G3, "prefill", B, S, T, dynamic_prefill=dyn)
        outs.append(interp.run_mlir(shlo.graph_to_mlir_text(g), [x, pos] + w + kv))
    for a, b in zip(outs[0], outs[1]):
        rms = float(np.sqrt(np.mean(np.square(b.astype(np.float64))))) + 1e-30
        assert approx_equal(a, b, atol=2e-2 * rms, rtol=2e-2)


def test_decode_step_continues_prefill():
    """Prefill S tokens then decode 1 equals prefill of S+1 tokens at the last row."""
    B, S, T = 1, 6, 16
    cfg = TINY_G3
    w = d.make_weights(cfg)
    toks = d.make_prompt(cfg, B, S + 1)
    kv = [d.zero_cache(cfg, B, T) for _ in range(2 * cfg.layers)]
    gp = shlo.graph_to_mlir_text(d.build_graph(cfg, "prefill", B, S, T))
    gd = shlo.graph_to_mlir_text(d.build_graph(cfg, "decode", B, S, T))
    out = interp.run_mlir(gp, [toks[:, :S], d.pos_inputs(cfg, "prefill", B, 0, S)] + w + kv)
    out2 = interp.run_mlir(gd, [toks[:, S:S + 1], d.pos_inputs(cfg, "decode", B, S, 1)] + w + list(out[1:]))
    gfull = shlo.graph_to_mlir_text(d.build_graph(cfg, "prefill", B, S + 1, T))
    ref = interp.run_mlir(gfull, [toks, d.pos_inputs(cfg, "prefill", B, 0, S + 1)] + w + kv)
    a, b = out2[0][0, 0], ref[0][0, S]
    rms = float(np.sqrt(np.mean(np.square(b.astype(np.float64)))))
    assert approx_equal(a, b, atol=5e-2 * rms, rtol=5e-2)


def test_ulp_noise_is_summation_order_sized():
    """The noise-floor option of the oracle perturbs f32 dot results by a few
    ulps (normal, sigma sqrt(K)/5 with K = 64 here: at least one ulp, rarely
    more than 5), and leaves non-accumulating ops untouched."""
    g = t.trace_graph("nz", [("a", ("tensor", (4, 64), "f32")), ("b", ("tensor", (64, 32), "f32"))],
                      lambda a, b: [t.matmul(a, b), t.add(a, a)])
    text = shlo.graph_to_mlir_text(g)
    rng = np.random.Generator(np.random.PCG64(0))
    a = rng.standard_normal((4, 64)).astype(np.float32)
    b = rng.standard_normal((64, 32)).astype(np.float32)
    base = interp.run_mlir(text, [a, b])
    noisy = interp.run_mlir(text, [a, b], ulp_noise_seed=5)
    gap = np.abs(noisy[0].astype(np.float64) - base[0]) / np.spacing(np.abs(base[0]))
    assert gap.max() <= 6.0 + 1e-9 and (gap > 0).any() and np.median(gap) <= 2.0
    np.testing.assert_array_equal(noisy[1], base[1])
