"""Per-op parity on the B200: each printed op form, run through the PJRT C ABI
of libcljxla_b200.so, against the numpy oracle on the same seeded inputs.

Graphs are traced with the host mirror of clj-xla's tensor API
(src/clj_xla/tensor.clj), so every MLIR form comes from the reference printer
rules (src/clj_xla/stablehlo.clj).
"""
import numpy as np
import pytest

from cljxla_b200.host import core, runner
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


def rand(shape, dt, seed=0, scale=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    if dt == "i32":
        return rng.integers(0, 7, size=shape, dtype=np.int64).astype(np.int32)
    a = (rng.standard_normal(shape) * scale).astype(np.float32)
    return interp.f32_to_bf16_bits(a) if dt == "bf16" else a


def check_graph(ctx, g, inputs, rtol=None):
    text = shlo.graph_to_mlir_text(g)
    want = interp.run_mlir(text, inputs)
    got = runner.run_graph(ctx, g, inputs, text)
    specs = runner.out_specs(g)
    for i, ((shape, dt), a, b) in enumerate(zip(specs, got, want)):
        assert tuple(a.shape) == tuple(shape)
        ok, excess, maxerr = close(a, b, dt, rtol)
        assert ok, f"output {i} ({dt}{shape}) differs: max err {maxerr}, excess {excess}"
    return got


def test_reference_known_answer_on_gpu(ctx):
    # rocm_e2e_test.clj:38-51: y = 2.5 x for x = 0..15 within 1e-4
    g = {"name": "parity_test_graph", "invars": [("x", ("tensor", (1, 16), "f32"))], "outvars": ["y"],
         "eqns": [{"op": "stablehlo/constant", "value": 2.5, "outvars": ["c0"]},
                  {"op": "stablehlo/multiply", "invars": ["x", "c0"], "outvars": ["y"]}]}
    x = np.arange(16, dtype=np.float32).reshape(1, 16)
    (y,) = runner.run_graph(ctx, g, [x])
    np.testing.assert_allclose(y.ravel(), 2.5 * np.arange(16), atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_elementwise_chain(ctx, dt):
    def f(x, y):
        a = t.add(t.mul(x, 2.0), y)
        b = t.div(t.exp(t.sub(a, 1.0)), t.add(t.tanh(y), 3.0))
        return [t.sqrt(t.add(t.mul(b, b), 1e-3)), t.sin(x), t.cos(y), t.maximum(x, y), t.sigmoid(a)]
    g = t.trace_graph("ew", [("x", ("tensor", (3, 5, 7), dt)), ("y", ("tensor", (3, 5, 7), dt))], f)
    check_graph(ctx, g, [rand((3, 5, 7), dt, 1), rand((3, 5, 7), dt, 2)])


def test_broadcast_convert_compare_select(ctx):
    def f(x, v, s):
        xb = t.mul(x, v)                       # [4,6] * [6] -> broadcast_in_dim
        c = t.compare_t(xb, t.convert(s, "f32"), "GT")
        return [t.select(c, xb, t.sub(xb)), t.convert(xb, "bf16"), t.convert(t.convert(x, "i32"), "f32")]
    g = t.trace_graph("bcs", [("x", ("tensor", (4, 6), "f32")), ("v", ("tensor", (6,), "f32")),
                              ("s", ("tensor", (4, 6), "i32"))], f)
    check_graph(ctx, g, [rand((4, 6), "f32", 3, 3.0), rand((6,), "f32", 4), rand((4, 6), "i32", 5)])


def test_reshape_transpose_slice_concat(ctx):
    def f(x):
        r = t.transpose(t.reshape(x, [2, 3, 4, 5]), [0, 2, 1, 3])
        s = t.slice(r, [0, 1, 0, 1], [2, 4, 3, 5], [1, 1, 1, 2])
        c = t.concatenate([t.sub(s), s], -1)
        return [c, t.reshape(t.transpose(r, [0, 2, 1, 3]), [6, 20])]
    g = t.trace_graph("mv", [("x", ("tensor", (6, 20), "bf16"))], f)
    check_graph(ctx, g, [rand((6, 20), "bf16", 6)])


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_reductions_and_argmax(ctx, dt):
    def f(x):
        return [t.reduce_sum(x, axes=[-1]), t.reduce_max(x, axes=[1], keep_dims=False),
                t.reduce_mean(t.pow(x, 2.0), axes=[-1]), t.argmax(x)]
    g = t.trace_graph("red", [("x", ("tensor", (3, 50, 300), dt))], f)
    check_graph(ctx, g, [rand((3, 50, 300), dt, 7)])


@pytest.mark.parametrize("dt,rows,V", [("f32", 3, 262144), ("bf16", 8, 262144), ("bf16", 2, 1000)])
def test_argmax_kernel_with_planted_ties(ctx, dt, rows, V):
    """The printed argmax (tensor.clj:519-532) runs as one kernel (rows split
    over CTAs at vocabulary size); the token ids equal the oracle's bit for bit,
    including the highest-index rule for ties planted across CTA boundaries,
    for f32 logits and for bf16 logits widened to f32 as the Gemma graphs print."""
    def f(x):
        return [t.argmax(t.convert(x, "f32") if dt == "bf16" else x)]
    g = t.trace_graph("amax", [("x", ("tensor", (rows, 1, V), dt))], f)
    text = shlo.graph_to_mlir_text(g)
    exe = core.compile_mlir_text(ctx, text, g)
    assert core.plan_info(ctx, exe)["launches"] <= 2  # the argmax kernel (+ the reshaped result)
    x = interp.bf16_bits_to_f32(rand((rows, 1, V), "bf16", 31)) if dt == "bf16" else rand((rows, 1, V), "f32", 31)
    x = np.array(x, np.float32)
    for r in range(rows):  # the same maximum at indices far apart
        top = np.float32(9.0 + r)
        for j in (5 * r, V // 3 + r, V - 1 - 7 * r):
            x[r, 0, j] = top
    inp = interp.f32_to_bf16_bits(x) if dt == "bf16" else x
    want = interp.run_mlir(text, [inp])[0]
    got = runner.run_graph(ctx, g, [inp], text)[0]
    assert got.dtype == np.int32 and np.array_equal(got, want), (got.ravel(), want.ravel())
    assert np.array_equal(got.ravel(), [V - 1 - 7 * r for r in range(rows)])


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_dot_general_forms(ctx, dt):
    def f(x, w, q, k):
        lin = t.matmul(x, w)                                                    # [2,5,64]x[64,48]
        nt = t.dot_general(x, t.transpose(t.transpose(w, [1, 0]), [1, 0]),
                           {"contracting_dims": {"lhs": [2], "rhs": [0]}})
        sc = t.dot_general(q, k, {"batch_dims": {"lhs": [0, 1], "rhs": [0, 1]},
                                  "contracting_dims": {"lhs": [3], "rhs": [3]}})
        pv = t.dot_general(t.convert(sc, "f32"), k, {"batch_dims": {"lhs": [0, 1], "rhs": [0, 1]},
                                                     "contracting_dims": {"lhs": [3], "rhs": [2]}})
        return [lin, nt, sc, pv]
    g = t.trace_graph("dot", [("x", ("tensor", (2, 5, 64), dt)), ("w", ("tensor", (64, 48), dt)),
                              ("q", ("tensor", (1, 4, 3, 32), dt)), ("k", ("tensor", (1, 4, 9, 32), dt))], f)
    check_graph(ctx, g, [rand((2, 5, 64), dt, 8, 0.5), rand((64, 48), dt, 9, 0.5),
                         rand((1, 4, 3, 32), dt, 10, 0.5), rand((1, 4, 9, 32), dt, 11, 0.5)])


@pytest.mark.parametrize("M,K,N", [(1, 768, 2304), (1, 768, 3072), (1, 3072, 768), (3, 768, 1000), (8, 256, 520)])
def test_few_row_f32_products(ctx, M, K, N):
    """f32 x [M, K] against f32 weights in both layouts GPT-2 decode uses:
    [K, N] (Conv1D, N contiguous) and transpose([N, K]) (the tied LM head),
    on the few-row kernels that stream each weight once."""
    def f(x, w, v):
        return [t.matmul(x, w), t.matmul(x, t.transpose(v, [1, 0]))]
    g = t.trace_graph("f32rows", [("x", ("tensor", (M, K), "f32")), ("w", ("tensor", (K, N), "f32")),
                                  ("v", ("tensor", (N, K), "f32"))], f)
    check_graph(ctx, g, [rand((M, K), "f32", 21, 0.5), rand((K, N), "f32", 22, 0.05), rand((N, K), "f32", 23, 0.05)])


def test_large_dense_literal(ctx):
    """A dense literal of 400 K values (about 5 MB of printed text, the size of
    a static-position prefill mask) is parsed in chunks on several host threads
    and through the exact decimal fast path: every value equals the oracle's."""
    n = 400_000
    rng = np.random.Generator(np.random.PCG64(31))
    vals = (rng.standard_normal(n) * 10.0 ** rng.integers(-6, 6, n)).astype(np.float32)
    vals[::7] = -10000.0
    vals[::11] = 0.0
    g = t.trace_graph("biglit", [("x", ("tensor", (n,), "f32"))],
                      lambda x: [t.add(x, t.emit_constant([float(v) for v in vals], ("tensor", (n,), "f32")))])
    text = shlo.graph_to_mlir_text(g)
    assert len(text) > 4 << 20
    x = np.zeros(n, np.float32)
    got = runner.run_graph(ctx, g, [x], text)[0]
    want = interp.run_mlir(text, [x])[0]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_gather_rows_and_clamp(ctx):
    def f(tab, ids):
        return t.gather(tab, ids)
    g = t.trace_graph("gth", [("tab", ("tensor", (50, 24), "bf16")), ("ids", ("tensor", (2, 7), "i32"))], f)
    ids = np.array([[0, 5, 49, 50, 1000, -3, 7], [1, 2, 3, 4, 5, 6, 7]], np.int32)
    inputs = [rand((50, 24), "bf16", 12), ids]
    got = check_graph(ctx, g, inputs)
    # row copies are bit-exact: same bf16 bit patterns as the oracle's clamped rows
    want = interp.f32_to_bf16_bits(interp.run_mlir(shlo.graph_to_mlir_text(g), inputs)[0])
    assert got[0].dtype == np.uint16 and np.array_equal(got[0], want)
    rows = np.clip(ids, 0, 49)
    assert np.array_equal(got[0], inputs[0][rows])


def test_dynamic_update_slice_tracer_and_constant_index(ctx):
    def f(cache, new, pos):
        return [t.dynamic_update_slice(cache, new, [0, 0, pos, 0]),
                t.dynamic_update_slice(cache, new, [0, 1, 3, 0])]
    g = t.trace_graph("dus", [("c", ("tensor", (1, 2, 16, 8), "bf16")), ("n", ("tensor", (1, 2, 1, 8), "bf16")),
                              ("p", ("tensor", (1,), "i32"))], f)
    for p in (0, 5, 15, 40):   # 40 is clamped to 15 (StableHLO semantics)
        check_graph(ctx, g, [rand((1, 2, 16, 8), "bf16", 13), rand((1, 2, 1, 8), "bf16", 14),
                             np.array([p], np.int32)])


def test_iota_mask_path(ctx):
    from cljxla_b200.host import nn

    def f(pos):
        return nn.generate_causal_mask(4, 12, pos, 3)
    g = t.trace_graph("mask", [("pos", ("tensor", (1,), "i32"))], f)
    for p in (0, 5):
        check_graph(ctx, g, [np.array([p], np.int32)])


def test_compile_errors_are_pjrt_errors(ctx):
    from cljxla_b200.host.pjrt import PJRTError
    with pytest.raises(PJRTError) as e:
        ctx["api"].compile_mlir(ctx["client"], "module @bad {\n  func.func @main(%x: tensor<2xf32>) -> (tensor<2xf32>) {\n    %y = stablehlo.foo %x : tensor<2xf32>\n    return %y : tensor<2xf32>\n  }\n}\n")
    assert e.value.code == 12  # UNIMPLEMENTED
    with pytest.raises(PJRTError) as e:
        ctx["api"].compile_mlir(ctx["client"], "module @bad {\n garbage\n}\n")
    assert e.value.code == 3   # INVALID_ARGUMENT


def test_execute_argument_mismatch_is_error(ctx):
    from cljxla_b200.host.pjrt import PJRTError
    g = t.trace_graph("m", [("x", ("tensor", (2, 3), "f32"))], lambda x: t.mul(x, 2.0))
    exe = core.compile_graph(ctx, g)
    b = core.buffer_from_host_buffer(ctx, np.zeros((3, 2), np.float32), [3, 2], 11)
    with pytest.raises(PJRTError) as e:
        ctx["api"].execute_executable(exe["handle"], [b], 1)
    assert e.value.code == 3
    core.destroy_buffer(ctx, b)


def test_compile_cache_returns_identical_handle(ctx):
    # compile_test.clj:7-21
    core.clear_cache()
    g = {"name": "cached_graph", "invars": [("x", ("tensor", (2, 32), "f32"))], "outvars": ["y"],
         "eqns": [{"op": "stablehlo/constant", "value": 3.0, "outvars": ["c0"]},
                  {"op": "stablehlo/multiply", "invars": ["x", "c0"], "outvars": ["y"]}]}
    e1 = core.compile_graph(ctx, g)
    e2 = core.compile_graph(ctx, g)
    assert e1["handle"] == e2["handle"]


def test_platform_and_single_device(ctx):
    assert ctx["platform"] == "cuda"
    assert len(ctx["api"].addressable_devices(ctx["client"])) == 1


def test_large_upload_through_pinned_staging_is_exact(ctx):
    """Uploads of 8 MiB and more go through the pinned staging ring in 32 MiB
    chunks (weight ingest); a ragged size spanning three chunks, and a second
    buffer reusing the ring, read back bit for bit."""
    from cljxla_b200.host.pjrt import DTYPE_ENUM
    rng = np.random.Generator(np.random.PCG64(21))
    for n in (17_000_003, 2_500_000):
        a = rng.standard_normal(n, dtype=np.float32)
        b = core.buffer_from_host_buffer(ctx, a, (n,), DTYPE_ENUM["f32"])
        try:
            got = core.buffer_to_numpy(ctx, b, (n,), "f32")
        finally:
            core.destroy_buffer(ctx, b)
        assert np.array_equal(got.view(np.uint32), a.view(np.uint32))


def test_memory_limit_gives_resource_exhausted(ctx):
    """A client created with memory_limit_bytes refuses allocations past it
    with PJRT RESOURCE_EXHAUSTED (code 8) - uploads and execution outputs
    alike - and accepts them again once buffers are released."""
    from cljxla_b200.host.pjrt import DTYPE_ENUM, PJRTError
    api = ctx["api"]
    client = api.create_client({"memory_limit_bytes": 64 << 20})
    c2 = core.Context(ctx, client=client)
    try:
        _memory_limit_checks(api, c2, DTYPE_ENUM["f32"], PJRTError)
    finally:
        core.close_backend(c2)


def _memory_limit_checks(api, c2, f32, PJRTError):
    a = np.ones(8 << 20, np.float32)           # 32 MiB
    b1 = core.buffer_from_host_buffer(c2, a, a.shape, f32)
    with pytest.raises(PJRTError) as e:
        core.buffer_from_host_buffer(c2, np.ones(10 << 20, np.float32), (10 << 20,), f32)  # 40 MiB more
    assert e.value.code == 8 and "RESOURCE_EXHAUSTED" in str(e.value)
    g = t.trace_graph("twice", [("x", ("tensor", (8 << 20,), "f32"))], lambda x: [t.add(x, x)])
    exe = core.compile_mlir_text(c2, shlo.graph_to_mlir_text(g), g)
    out = api.execute_executable(exe["handle"], [b1], 1)    # 32 + 32 MiB: at the cap, allowed
    with pytest.raises(PJRTError) as e:
        api.execute_executable(exe["handle"], [b1], 1)      # a third 32 MiB is not
    assert e.value.code == 8
    core.destroy_buffer(c2, out)
    out = api.execute_executable(exe["handle"], [b1], 1)    # released memory counts again
    assert np.array_equal(core.buffer_to_numpy(c2, out, (8 << 20,), "f32"), 2 * a)
    core.destroy_buffer(c2, out)
    core.destroy_buffer(c2, b1)
