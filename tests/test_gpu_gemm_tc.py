"""The tensor-core (tcgen05) GEMM on prefill-shaped linear layers.

Gemma's linear layer is dot_general(x[.., K], W[N, K]) contracting the
weight's last dim when N != K (gemma.clj:8-23), bf16 operands; the planner
sends the ones with more than 8 rows to the tcgen05 kernel (128 x 256 tiles,
or 64-wide weight tiles with K split over CTAs for at most 128 rows).  Each case checks that the kernel actually ran (profile entries of kind
gemm_tc) and compares with the numpy oracle at the bf16 tolerance; ragged M / N
/ K exercise the TMA zero-filled tile edges and the guarded epilogue.
"""
import dataclasses

import numpy as np
import pytest

from cljxla_b200.host import core, drivers as d, runner
from cljxla_b200.host import models
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200.host import tensor as t
from oracle import interp

from conftest import has_gpu
from parity import close, close_model_floor

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    if not has_gpu():
        pytest.skip("no CUDA device")
    from cljxla_b200 import LIB_PATH
    return core.init_backend(LIB_PATH)


def _bf16(shape, seed, scale=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    return interp.f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def _run_profiled(ctx, g, inputs, text):
    core.profile_enable(ctx, True)
    try:
        got = runner.run_graph(ctx, g, inputs, text)
        prof = core.profile_dump(ctx)
    finally:
        core.profile_enable(ctx, False)
    return got, prof


@pytest.mark.parametrize("S,K,N", [
    (128, 256, 192),     # one tile (N != K: gemma_linear contracts the weight's last dim)
    (200, 320, 300),     # ragged M, N and a K tail inside one 64-wide block
    (17, 64, 40),        # smaller than a tile
    (512, 2560, 1024),   # Gemma-3-4B k/v projection shape, four M tiles
    (256, 1024, 2304),   # N spans nine 256-wide tiles
    # a few rows (batched decode): 64-wide weight tiles, K split over CTAs
    (32, 2304, 2048),    # Gemma-2-2B batch-32 q projection: 32 tiles x 4 K splits
    (9, 2304, 1000),     # 9 rows (A copies of 16 rows), ragged N inside a 64-wide tile
    (16, 5376, 512),     # Gemma-3-27B TP8 shard: 8 tiles x 18 K splits
    (100, 704, 2560),    # more than 64 rows: 256-wide tiles, 10 tiles x 2 K splits
])
def test_linear_layer_on_tensor_cores(ctx, S, K, N):
    g = t.trace_graph("tc_linear", [("x", ("tensor", (1, S, K), "bf16")), ("w", ("tensor", (N, K), "bf16"))],
                      lambda x, w: [models.gemma_linear(x, w)])
    text = shlo.graph_to_mlir_text(g)
    inputs = [_bf16((1, S, K), 1), _bf16((N, K), 2, 0.05)]
    want = interp.run_mlir(text, inputs)
    got, prof = _run_profiled(ctx, g, inputs, text)
    assert any(e["kind"] == "gemm_tc" for e in prof), [e["kind"] for e in prof]
    ok, excess, maxerr = close(got[0], want[0], "bf16")
    assert ok, f"max err {maxerr:.3g}, excess {excess:.3g}"


def test_repeated_runs_and_new_operands(ctx):
    """Graph replay with the same buffers, then new weight buffers (tensor maps re-encoded)."""
    S, K, N = 160, 512, 384
    g = t.trace_graph("tc_repeat", [("x", ("tensor", (1, S, K), "bf16")), ("w", ("tensor", (N, K), "bf16"))],
                      lambda x, w: [models.gemma_linear(x, w)])
    text = shlo.graph_to_mlir_text(g)
    for seed in (3, 4, 5):
        inputs = [_bf16((1, S, K), seed), _bf16((N, K), seed + 10, 0.05)]
        want = interp.run_mlir(text, inputs)
        for _ in range(2):
            got = runner.run_graph(ctx, g, inputs, text)
            assert close(got[0], want[0], "bf16")[0]


def test_gemma3_prefill_through_tensor_cores(ctx):
    cfg = dataclasses.replace(d.GEMMA3_4B, vocab=512, d_model=256, layers=2, n_heads=4, n_kv_heads=2,
                              head_dim=64, mlp=512, window=16)
    B, S, T = 1, 48, 64
    g = d.build_graph(cfg, "prefill", B, S, T, dynamic_prefill=True)
    text = shlo.graph_to_mlir_text(g)
    inputs = [d.make_prompt(cfg, B, S), d.pos_inputs(cfg, "prefill", B, 0, S)] + d.make_weights(cfg) + \
        [d.zero_cache(cfg, B, T) for _ in range(2 * cfg.layers)]
    want = interp.run_mlir(text, inputs)
    got, prof = _run_profiled(ctx, g, inputs, text)
    # k, v, gate, up, down per layer (q / o are square here, o's lhs is f32) and the LM head
    assert sum(e["calls"] for e in prof if e["kind"] == "gemm_tc") >= 5 * cfg.layers + 1
    floors = None
    for i, ((shape, dt), a, b) in enumerate(zip(runner.out_specs(g), got, want)):
        edt = "bf16" if dt == "f32" else dt
        if floors is None:
            floors = [interp.run_mlir(text, inputs, ulp_noise_seed=sd) for sd in (1, 2, 3, 4)]
        ok, bad, rr, fb, fr = close_model_floor(a, b, [f[i] for f in floors], edt)
        assert ok, f"output {i}: {bad:.2%} out of bound, rel rms {rr:.3g} (floor {fb:.2%}, {fr:.3g})"


def _f32(shape, seed, scale=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.standard_normal(shape) * scale).astype(np.float32)


@pytest.mark.parametrize("S,K,N", [
    (128, 256, 192),
    (200, 320, 300),     # ragged M / N: plane tiles read into the next plane's rows
    (512, 2048, 640),
    (32, 2048, 2304),    # a few rows: 64-wide tiles, K blocks of the three planes split over CTAs
    (20, 512, 300),
])
def test_f32_activation_times_bf16_weight_on_tensor_cores(ctx, S, K, N):
    """f32 x bf16 -> f32 (the attention-output projection of a Gemma prefill,
    gemma.clj attention block): the activation is split exactly into three bf16
    planes and the tcgen05 GEMM accumulates the three products, so the result
    matches the f32 oracle at the f32 tolerance."""
    g = t.trace_graph("tc_split", [("x", ("tensor", (1, S, K), "f32")), ("w", ("tensor", (N, K), "bf16"))],
                      lambda x, w: [models.gemma_linear(x, w)])
    text = shlo.graph_to_mlir_text(g)
    inputs = [_f32((1, S, K), 7), _bf16((N, K), 8, 0.05)]
    want = interp.run_mlir(text, inputs)
    got, prof = _run_profiled(ctx, g, inputs, text)
    kinds = [e["kind"] for e in prof]
    assert "gemm_tc" in kinds and "gemm_generic" not in kinds, kinds
    ok, excess, maxerr = close(got[0], want[0], "f32")
    assert ok, f"max err {maxerr:.3g}, excess {excess:.3g}"


def test_split_planes_read_through_head_merge(ctx):
    """The attention context [1, heads, S, hd] f32, transposed and reshaped to
    [1, S, heads * hd] as printed before the output projection: the planes are
    written straight from the permuted view (no materialised copy)."""
    H, S, hd, N = 4, 96, 64, 320
    def f(x, w):
        y = t.reshape(t.transpose(x, [0, 2, 1, 3]), [1, S, H * hd])
        return [models.gemma_linear(y, w)]
    g = t.trace_graph("tc_split_view", [("x", ("tensor", (1, H, S, hd), "f32")), ("w", ("tensor", (N, H * hd), "bf16"))], f)
    text = shlo.graph_to_mlir_text(g)
    inputs = [_f32((1, H, S, hd), 9), _bf16((N, H * hd), 10, 0.05)]
    want = interp.run_mlir(text, inputs)
    got, prof = _run_profiled(ctx, g, inputs, text)
    kinds = [e["kind"] for e in prof]
    assert "gemm_tc" in kinds and "copy" not in kinds, kinds
    ok, excess, maxerr = close(got[0], want[0], "f32")
    assert ok, f"max err {maxerr:.3g}, excess {excess:.3g}"
