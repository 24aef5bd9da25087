"""Computed attention masks on the B200.

The planner proves the printed causal / sliding-window mask
(attention.clj:189-224) equal to a closed form, and the attention kernels then
compute each mask value from the position instead of reading it.  The values
are the same f32 numbers (0 or -10000), so the plan with computed masks must
give bit-identical results to the plan that reads them
(``CLJXLA_B200_MASK_FORM=0``).  The cases cover every attention kernel the
mask reaches: the staged bf16 decode kernel (batch 1 and 4), the tensor-core
decode kernel, the f32 SIMT kernels (GPT-2), and the tensor-core prefill with
its fast path (a closed-form score chain) and without it (Gemma-2's softcap),
for the traced-position chain and the static literal, at positions where the
sliding window masks.
"""
import dataclasses

import numpy as np
import pytest

from cljxla_b200.host import core, drivers as d, runner
from cljxla_b200.host import stablehlo as shlo

from conftest import has_gpu

pytestmark = pytest.mark.gpu

TINY = {
    "gpt2": dataclasses.replace(d.GPT2_SMALL, vocab=384, d_model=384, layers=2, n_heads=12, n_kv_heads=12,
                                head_dim=32, mlp=768, n_positions=128),
    "gemma2": dataclasses.replace(d.GEMMA2_2B, vocab=512, d_model=256, layers=2, n_heads=4, n_kv_heads=2,
                                  head_dim=64, mlp=512, window=6),
    "gemma3": dataclasses.replace(d.GEMMA3_4B, vocab=512, d_model=256, layers=6, n_heads=4, n_kv_heads=2,
                                  head_dim=64, mlp=512, window=6),
}

# (family, kind, dynamic prefill, batch, prompt / position, cache length, extra planner switches)
CASES = [
    ("gemma3", "decode", False, 1, 20, 32, {}),                          # staged decode
    ("gemma3", "decode", False, 4, 27, 64, {}),
    ("gemma3", "decode", False, 2, 20, 32, {"CLJXLA_B200_ATTN_DEC": "0"}),  # tensor-core decode
    ("gemma2", "decode", False, 1, 13, 32, {}),
    ("gpt2", "decode", False, 1, 20, 32, {}),
    ("gemma3", "prefill", False, 1, 80, 96, {}),                         # literal mask, fast path
    ("gemma3", "prefill", True, 1, 80, 96, {}),                          # traced position
    ("gemma2", "prefill", True, 1, 80, 96, {}),                          # softcap: general chain
    ("gpt2", "prefill", False, 1, 12, 32, {}),
    ("gpt2", "prefill", True, 1, 12, 32, {}),
]


@pytest.fixture(scope="module")
def ctx():
    if not has_gpu():
        pytest.skip("no CUDA device")
    from cljxla_b200 import LIB_PATH
    return core.init_backend(LIB_PATH)


def _cache(cfg, B, T, seed):
    """A filled KV cache (N(0, 1) values) so every position's K / V matters."""
    rng = np.random.Generator(np.random.PCG64(seed))
    a = rng.standard_normal(d.cache_shape(cfg, B, T), dtype=np.float32)
    return d._to_bf16_bits(a) if cfg.dtype == "bf16" else a


def _run(ctx, graph, text, inputs):
    handle = ctx["api"].compile_mlir(ctx["client"], text)   # not the host cache: the switch acts at planning
    try:
        info = core.plan_info(ctx, {"handle": handle})
        bufs = runner.upload(ctx, graph, inputs)
        try:
            outs = ctx["api"].execute_executable(handle, bufs, len(graph["outvars"]))
            outs = outs if isinstance(outs, list) else [outs]
            res = []
            for b, (shape, dt) in zip(outs, runner.out_specs(graph)):
                res.append(core.buffer_to_numpy(ctx, b, shape, dt))
                core.destroy_buffer(ctx, b)
            return info, res
        finally:
            for b in bufs:
                core.destroy_buffer(ctx, b)
    finally:
        ctx["api"].destroy_executable(handle)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[1]}{'-dyn' if c[2] else ''}-b{c[3]}-p{c[4]}"
                         + ("-" + "-".join(c[6]) if c[6] else ""))
def test_computed_mask_is_bit_exact(ctx, monkeypatch, case):
    family, kind, dynamic, B, P, T, env = case
    cfg = TINY[family]
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    # the staged decode kernel spreads the live positions of a computed mask over
    # its splits (another summation grouping, checked against the oracle in the
    # model tests); here both plans split [0, T) alike
    monkeypatch.setenv("CLJXLA_B200_ATTN_LIVE_SPLITS", "0")
    n = P if kind == "prefill" else 1
    graph = d.build_graph(cfg, kind, B, P, T, dynamic_prefill=dynamic)
    text = shlo.graph_to_mlir_text(graph)
    toks = d.make_prompt(cfg, B, n, seed=7)
    pos = d.pos_inputs(cfg, kind, B, 0 if kind == "prefill" else P, n)
    inputs = [toks, pos] + d.make_weights(cfg) + [_cache(cfg, B, T, 100 + i) for i in range(2 * cfg.layers)]
    monkeypatch.delenv("CLJXLA_B200_MASK_FORM", raising=False)
    on_info, on = _run(ctx, graph, text, inputs)
    monkeypatch.setenv("CLJXLA_B200_MASK_FORM", "0")
    off_info, off = _run(ctx, graph, text, inputs)
    assert on_info["computed_masks"] == cfg.layers and off_info["computed_masks"] == 0
    assert len(on) == len(off)
    for i, (a, b) in enumerate(zip(on, off)):
        assert a.dtype == b.dtype and a.shape == b.shape
        ok = np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(b).view(np.uint8))
        assert ok, f"output {i}: computed and read masks differ ({np.sum(a != b)} elements)"


@pytest.mark.parametrize("family,pos", [("gemma3", 300), ("gemma3", 511), ("gemma2", 200)])
def test_live_splits_match_oracle(ctx, monkeypatch, family, pos):
    """Staged decode over a 512-position cache (8 splits of 64 positions):
    with a computed mask the splits share only the live positions (the
    window on local layers, [0, pos] on global ones), and the decode step
    still equals the oracle's."""
    from oracle import interp
    from test_gpu_models import _compare_all
    cfg = TINY[family]
    B, T = 1, 512
    monkeypatch.delenv("CLJXLA_B200_ATTN_LIVE_SPLITS", raising=False)
    monkeypatch.delenv("CLJXLA_B200_MASK_FORM", raising=False)
    graph = d.build_graph(cfg, "decode", B, pos, T)
    text = shlo.graph_to_mlir_text(graph)
    toks = d.make_prompt(cfg, B, 1, seed=9)
    inputs = [toks, d.pos_inputs(cfg, "decode", B, pos, 1)] + d.make_weights(cfg) + \
        [_cache(cfg, B, T, 200 + i) for i in range(2 * cfg.layers)]
    info, got = _run(ctx, graph, text, inputs)
    assert info["computed_masks"] == cfg.layers
    want = interp.run_mlir(text, inputs)
    _compare_all(got, want, runner.out_specs(graph), f"{family} decode at {pos}, live splits", cfg.dtype,
                 lambda sd: interp.run_mlir(text, inputs, ulp_noise_seed=sd))
