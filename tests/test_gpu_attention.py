"""The attention block printed by gqa-causal-attention / causal-self-attention
(attention.clj:227-375) in isolation: the library's fused kernel (and, with
fast kernels off, the generic path) against the numpy oracle."""
import numpy as np
import pytest

from cljxla_b200.host import core, nn, runner
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200.host import tensor as t
from oracle import interp

from conftest import has_gpu
from parity import close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    if not has_gpu():
        pytest.skip("no CUDA device")
    from cljxla_b200 import LIB_PATH
    return core.init_backend(LIB_PATH)


def _rand(shape, seed, scale=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    return interp.f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


@pytest.mark.parametrize("Sq,T,nq,nkv,softcap,window,dynamic,hd,pos", [
    (1, 16, 4, 2, None, None, True, 64, None),
    (1, 40, 4, 2, 50.0, 6, True, 64, None),
    (5, 16, 4, 2, None, None, True, 64, None),
    (8, 16, 4, 2, None, 6, True, 64, None),
    (8, 16, 4, 2, None, None, False, 64, None),
    (3, 24, 2, 2, 50.0, None, True, 64, None),
    (8, 128, 8, 4, None, None, True, 64, None),
    # decode over a long cache: many position splits, sliding window, rounds of 32 positions
    (1, 2560, 8, 4, None, 1024, True, 256, 2100),
    (1, 2560, 8, 4, None, None, True, 256, 2559),
    (1, 700, 8, 4, 50.0, 300, True, 128, 650),
    (4, 1200, 4, 2, None, None, True, 256, 900),
    # prefill on the tensor cores: 64 query vectors per CTA, causal chunks skipped
    (100, 128, 8, 4, None, None, True, 64, 20),
    (70, 96, 4, 1, 50.0, 24, True, 128, 0),
    (130, 160, 2, 2, None, None, False, 256, None),
    (64, 64, 8, 1, None, None, True, 64, 0),
    (200, 512, 8, 4, None, 64, True, 256, 300),
])
def test_attention_block(ctx, Sq, T, nq, nkv, softcap, window, dynamic, hd, pos):
    _check_attention(ctx, Sq, T, nq, nkv, softcap, window, dynamic, hd, pos)


@pytest.mark.parametrize("Sq,T,nq,nkv,window,hd", [
    (100, 128, 8, 4, None, 64),
    (70, 96, 4, 1, 24, 128),
])
def test_attention_prefill_simt_path(ctx, monkeypatch, Sq, T, nq, nkv, window, hd):
    """The CUDA-core prefill kernel (taken where the tensor-core one cannot run)
    on the same blocks."""
    monkeypatch.setenv("CLJXLA_B200_ATTN_TC", "0")
    core.clear_cache()  # the switch is read when a program is compiled
    try:
        _check_attention(ctx, Sq, T, nq, nkv, None, window, True, hd, 0)
    finally:
        core.clear_cache()


@pytest.mark.parametrize("Sq,T,nq,nkv,window,hd", [
    (130, 192, 8, 4, None, 256),
    (100, 128, 4, 2, 40, 128),
])
def test_attention_prefill_f32_queries(ctx, Sq, T, nq, nkv, window, hd):
    """f32 queries (the Gemma-3 prefill: RoPE in f32 feeds the score product):
    three exact bf16 parts on the tensor cores, the f32 tile in shared memory
    beside the K, V and mask tiles."""
    _check_attention(ctx, Sq, T, nq, nkv, None, window, True, hd, 0, qdt="f32")


def _check_attention(ctx, Sq, T, nq, nkv, softcap, window, dynamic, hd, pos, qdt="bf16"):
    B = 1

    def f(q, k, v, kc, vc, ow, pos):
        p = pos if dynamic else 0
        out, updated = nn.gqa_causal_attention(q, k, v, ow, nq, nkv, softcap, [kc, vc], p,
                                               {"scale": 0.125, "sliding-window": window})
        return [out, updated[0], updated[1]]
    g = t.trace_graph("attn", [("q", ("tensor", (B, Sq, nq * hd), qdt)), ("k", ("tensor", (B, Sq, nkv * hd), "bf16")),
                               ("v", ("tensor", (B, Sq, nkv * hd), "bf16")),
                               ("kc", ("tensor", (B, nkv, T, hd), "bf16")), ("vc", ("tensor", (B, nkv, T, hd), "bf16")),
                               ("ow", ("tensor", (nq * hd, nq * hd), "bf16")), ("pos", ("tensor", (1,), "i32"))], f)
    text = shlo.graph_to_mlir_text(g)
    if pos is None:
        pos = min(T - Sq, 3)
    pos = np.array([pos], np.int32) if dynamic else np.array([0], np.int32)
    q_in = _rand((B, Sq, nq * hd), 1)
    if qdt == "f32":
        q_in = np.random.Generator(np.random.PCG64(11)).standard_normal((B, Sq, nq * hd)).astype(np.float32)
    inputs = [q_in, _rand((B, Sq, nkv * hd), 2), _rand((B, Sq, nkv * hd), 3),
              _rand((B, nkv, T, hd), 4), _rand((B, nkv, T, hd), 5), _rand((nq * hd, nq * hd), 6, 0.05), pos]
    want = interp.run_mlir(text, inputs)
    got = runner.run_graph(ctx, g, inputs, text)
    floors = None
    for i, ((shape, dt), a, b) in enumerate(zip(runner.out_specs(g), got, want)):
        ok, excess, maxerr = close(a, b, dt)
        if not ok and dt == "f32" and not np.isnan(a).any():
            # the bf16 scores of this block round once per element: a valid f32
            # summation order different from the oracle's flips a few of those
            # roundings, and over a short window one flip moves an output by more
            # than the f32 tolerance.  Such a result must stay within twice the
            # spread of oracle runs with summation-order noise on every f32 sum.
            if floors is None:
                floors = [interp.run_mlir(text, inputs, ulp_noise_seed=s) for s in range(4)]
            spread = max(close(f[i], b, dt)[2] for f in floors)
            ok = maxerr <= 2.0 * spread
            excess = maxerr - 2.0 * spread
        assert ok, f"output {i} ({dt}{shape}) differs: max err {maxerr:.3g}, excess {excess:.3g}"
