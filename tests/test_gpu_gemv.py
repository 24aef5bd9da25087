"""Decode GEMV exactness on the B200: the Gemma linear-layer form
``x [M, K] . transpose(W [N, K])`` (gemma.clj:8-23) through libcljxla_b200.so,
against an f64 reference of the same bf16 inputs.  f32 results must agree to
f32 summation-order error; bf16 results may differ from the correctly rounded
value by at most one bf16 ulp (an f32 sum in another order can fall on the
other side of a rounding boundary), and only rarely.  Covers the shapes of the
Gemma decode projections, several projections of one input grouped into one
launch, f32 x, and batched rows (M > 1, on the tensor cores where K allows)."""
import numpy as np
import pytest

from cljxla_b200.host import core, runner
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200.host import tensor as t
from oracle import interp

from conftest import has_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    if not has_gpu():
        pytest.skip("no CUDA device")
    from cljxla_b200 import LIB_PATH
    return core.init_backend(LIB_PATH)


def _bf16(shape, seed, scale):
    rng = np.random.Generator(np.random.PCG64(seed))
    return interp.f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def _check(got, want64, dt):
    if dt == "f32":
        rms = float(np.sqrt(np.mean(want64 ** 2)))
        err = np.abs(got.astype(np.float64) - want64)
        assert err.max() <= 1e-5 * rms + 1e-6 * np.abs(want64).max(), err.max()
        return
    g = interp.bf16_bits_to_f32(got).astype(np.float64)
    ulp = np.spacing(np.abs(interp.bf16_bits_to_f32(interp.f32_to_bf16_bits(want64.astype(np.float32)))).astype(
        np.float32)).astype(np.float64) * 65536.0
    off = np.abs(g - want64)
    # plus f32 summation noise where a sum cancels to a value far below the
    # typical one (about 2^-17 of the RMS: an order above a K-term f32 sum's error)
    tol = ulp + 2.0 ** -17 * float(np.sqrt(np.mean(want64 ** 2)))
    worst = np.unravel_index(int(np.argmax(off / tol)), off.shape)
    assert (off <= tol).all(), (f"{float((off / tol).max()):.2f} x tolerance at {worst}: "
                                f"got {float(g[worst])!r} exact {float(want64[worst])!r}")
    # a flipped rounding needs the exact value within a few f32 ulps of a boundary: rare
    exact = interp.f32_to_bf16_bits(want64.astype(np.float32))
    assert np.mean(got != exact) < 0.01


@pytest.mark.parametrize("M,K,Ns,x_dt,out_dt", [
    (1, 2560, (2048, 1024, 1024), "bf16", "bf16"),   # Gemma-3-4B q / k / v
    (1, 2560, (10240, 10240), "bf16", "bf16"),       # gate / up
    (1, 10240, (2560,), "bf16", "bf16"),             # down
    (1, 2048, (2560,), "f32", "bf16"),               # o projection of the f32 attention output
    (1, 2560, (4096,), "bf16", "f32"),               # f32 result (logits)
    (1, 256, (256, 128, 128), "bf16", "bf16"),       # small test-model shapes
    (4, 3840, (512, 256), "bf16", "bf16"),           # batched decode rows (tensor cores)
    (8, 1024, (768,), "f32", "f32"),                 # f32 x as three bf16 parts
    (2, 2560, (2048, 1024, 1024), "bf16", "bf16"),
    (8, 3840, (7680, 7680), "bf16", "bf16"),         # Gemma-3-12B gate / up at TP2, batch 8
    (8, 2048, (3840,), "f32", "bf16"),               # its o projection
    (8, 7680, (3840,), "bf16", "bf16"),              # its down projection (K in chunks of the stage)
    (8, 15360, (3840,), "bf16", "bf16"),             # Gemma-3-12B down at TP1
    (8, 4096, (3840,), "f32", "bf16"),               # f32 x that does not fit shared memory whole
    (3, 5376, (1024,), "bf16", "f32"),
])
def test_decode_gemv_exact(ctx, M, K, Ns, x_dt, out_dt):
    def f(x, *ws):
        outs = []
        for w in ws:
            y = t.dot_general(x, t.transpose(w, [1, 0]), {"contracting_dims": {"lhs": [1], "rhs": [0]}})
            outs.append(t.convert(y, out_dt) if y.type[2] != out_dt else y)
        return outs
    inv = [("x", ("tensor", (M, K), x_dt))] + [(f"w{i}", ("tensor", (n, K), "bf16")) for i, n in enumerate(Ns)]
    g = t.trace_graph(f"gemv_{M}_{K}_{len(Ns)}_{x_dt}_{out_dt}", inv, f)
    text = shlo.graph_to_mlir_text(g)
    x = _bf16((M, K), 1, 1.0) if x_dt == "bf16" else np.random.default_rng(2).standard_normal((M, K)).astype(np.float32)
    ws = [_bf16((n, K), 10 + i, 0.02) for i, n in enumerate(Ns)]
    got = runner.run_graph(ctx, g, [x] + ws, text)
    xf = (interp.bf16_bits_to_f32(x) if x_dt == "bf16" else x).astype(np.float64)
    # the value is rounded once to bf16 when the dot's own result type (bf16 for
    # two bf16 operands, then converted) or the output is bf16
    for out, w, (shape, dt) in zip(got, ws, runner.out_specs(g)):
        want = xf @ interp.bf16_bits_to_f32(w).astype(np.float64).T
        check_dt = "bf16" if (x_dt == "bf16" or dt == "bf16") else "f32"
        if check_dt == "bf16" and dt == "f32":
            out = interp.f32_to_bf16_bits(out)  # exact: the values are bf16
        _check(out, want, check_dt)
