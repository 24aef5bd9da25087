"""KV-cache updates executed in place keep PJRT buffer semantics.

A decode step returns ``dynamic_update_slice(cache, new, pos)`` while the
caller still holds the old cache buffer (attention.clj:170-184 builds the
update; pjrt.clj:478-480 never donates inputs).  The library writes the new
row into the old buffer's storage and keeps the old buffer readable through an
undo record.  These tests check, bit for bit, that every buffer of a chain
still reads as its own value in any read/destroy order, that a stale buffer
can be passed back in, and that aliased arguments fall back to a copy.
"""
import numpy as np
import pytest

from cljxla_b200.host import core, nn
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200.host import tensor as t
from cljxla_b200.host.pjrt import DTYPE_ENUM
from oracle import interp

from conftest import has_gpu

pytestmark = pytest.mark.gpu

SHAPE = (1, 2, 16, 8)  # [batch, kv heads, max_seq, head_dim]


@pytest.fixture(scope="module")
def ctx():
    if not has_gpu():
        pytest.skip("no CUDA device")
    from cljxla_b200 import LIB_PATH
    return core.init_backend(LIB_PATH)


def step_graph(with_other=False):
    inv = [("cache", ("tensor", SHAPE, "bf16"))]
    if with_other:
        inv.append(("other", ("tensor", SHAPE, "bf16")))
    inv += [("new", ("tensor", (1, 2, 1, 8), "f32")), ("pos", ("tensor", (1,), "i32"))]

    def f(*a):
        cache, new, pos = a[0], a[-2], a[-1]
        updated, _ = nn._update_single_cache(cache, new, pos)
        src = a[1] if with_other else updated
        total = t.reduce_sum(t.convert(src, "f32"), axes=[-1])
        return [updated, total]

    return t.trace_graph("kv_step", inv, f)


def upload(ctx, a, shape, dt):
    return core.buffer_from_host_buffer(ctx, np.ascontiguousarray(a), shape, DTYPE_ENUM[dt])


def read_cache(ctx, buf):
    return core.buffer_to_numpy(ctx, buf, SHAPE, "bf16")


def rows(seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((1, 2, 1, 8)).astype(np.float32)


def apply(cache_bits, new, pos):
    out = cache_bits.copy()
    out[:, :, pos:pos + 1, :] = interp.f32_to_bf16_bits(new)
    return out


class Stepper:
    def __init__(self, ctx, with_other=False):
        self.ctx = ctx
        g = step_graph(with_other)
        self.exe = core.compile_mlir_text(ctx, shlo.graph_to_mlir_text(g), g)
        self.with_other = with_other

    def __call__(self, cache_buf, new, pos, other_buf=None):
        nb = upload(self.ctx, new, (1, 2, 1, 8), "f32")
        pb = upload(self.ctx, np.array([pos], np.int32), (1,), "i32")
        args = [cache_buf] + ([other_buf] if self.with_other else []) + [nb, pb]
        try:
            outs = self.ctx["api"].execute_executable(self.exe["handle"], args, 2)
        finally:
            core.destroy_buffer(self.ctx, nb)
            core.destroy_buffer(self.ctx, pb)
        total = core.buffer_to_numpy(self.ctx, outs[1], (1, 2, 16, 1), "f32")
        core.destroy_buffer(self.ctx, outs[1])
        return outs[0], total


def base_cache(seed=7):
    rng = np.random.Generator(np.random.PCG64(seed))
    return interp.f32_to_bf16_bits(rng.standard_normal(SHAPE).astype(np.float32))


def sums(bits):
    return interp.bf16_bits_to_f32(bits).astype(np.float64).sum(-1, keepdims=True)


def test_chain_every_version_readable(ctx):
    step = Stepper(ctx)
    c0 = base_cache()
    want = [c0]
    bufs = [upload(ctx, c0, SHAPE, "bf16")]
    for k in range(6):
        nb, total = step(bufs[-1], rows(k), k + 3)
        want.append(apply(want[-1], rows(k), k + 3))
        np.testing.assert_allclose(total, sums(want[-1]), rtol=1e-5, atol=1e-4)
        bufs.append(nb)
    # oldest first, then newest first: every buffer keeps its own content
    for b, w in zip(bufs, want):
        np.testing.assert_array_equal(read_cache(ctx, b), w)
    for b, w in reversed(list(zip(bufs, want))):
        np.testing.assert_array_equal(read_cache(ctx, b), w)
    for b in bufs:
        core.destroy_buffer(ctx, b)


@pytest.mark.parametrize("order", ["head_first", "middle_first", "oldest_first"])
def test_destroy_orders(ctx, order):
    step = Stepper(ctx)
    want = [base_cache(11)]
    bufs = [upload(ctx, want[0], SHAPE, "bf16")]
    for k in range(4):
        nb, _ = step(bufs[-1], rows(20 + k), 2 * k)
        want.append(apply(want[-1], rows(20 + k), 2 * k))
        bufs.append(nb)
    kill = {"head_first": [4, 2], "middle_first": [2, 3], "oldest_first": [0, 1]}[order]
    for i in kill:
        core.destroy_buffer(ctx, bufs[i])
    for i in range(5):
        if i not in kill:
            np.testing.assert_array_equal(read_cache(ctx, bufs[i]), want[i])
    for i in range(5):
        if i not in kill:
            core.destroy_buffer(ctx, bufs[i])


def test_stale_buffer_passed_back(ctx):
    step = Stepper(ctx)
    c0 = base_cache(3)
    b0 = upload(ctx, c0, SHAPE, "bf16")
    b1, _ = step(b0, rows(1), 0)
    b2, _ = step(b1, rows(2), 1)
    # b0 and b1 are stale now; stepping from them forks new chains
    f0, t0 = step(b0, rows(5), 9)
    f1, t1 = step(b1, rows(6), 15)
    w1 = apply(c0, rows(1), 0)
    w2 = apply(w1, rows(2), 1)
    wf0 = apply(c0, rows(5), 9)
    wf1 = apply(w1, rows(6), 15)
    np.testing.assert_allclose(t0, sums(wf0), rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(t1, sums(wf1), rtol=1e-5, atol=1e-4)
    for b, w in [(b0, c0), (b1, w1), (b2, w2), (f0, wf0), (f1, wf1)]:
        np.testing.assert_array_equal(read_cache(ctx, b), w)
    # continue the forked chain twice more (graph replay path)
    g1, _ = step(f1, rows(7), 4)
    g2, _ = step(g1, rows(8), 5)
    wg1 = apply(wf1, rows(7), 4)
    np.testing.assert_array_equal(read_cache(ctx, g2), apply(wg1, rows(8), 5))
    np.testing.assert_array_equal(read_cache(ctx, f1), wf1)
    for b in [b0, b1, b2, f0, f1, g1, g2]:
        core.destroy_buffer(ctx, b)


def test_long_chain_oldest_rebuilt(ctx):
    step = Stepper(ctx)
    c0 = base_cache(5)
    w = c0
    b0 = upload(ctx, c0, SHAPE, "bf16")
    cur = b0
    chain = []
    for k in range(40):
        nb, _ = step(cur, rows(100 + k), k % 16)
        w = apply(w, rows(100 + k), k % 16)
        if cur is not b0:
            chain.append(cur)
        cur = nb
    np.testing.assert_array_equal(read_cache(ctx, b0), c0)
    np.testing.assert_array_equal(read_cache(ctx, cur), w)
    for b in chain + [b0, cur]:
        core.destroy_buffer(ctx, b)


def test_aliased_arguments_are_not_updated_in_place(ctx):
    step = Stepper(ctx, with_other=True)
    c0 = base_cache(9)
    b0 = upload(ctx, c0, SHAPE, "bf16")
    # the same buffer as cache and as the independent operand: the update must not leak into it
    b1, total = step(b0, rows(1), 4, other_buf=b0)
    np.testing.assert_allclose(total, sums(c0), rtol=1e-5, atol=1e-4)
    np.testing.assert_array_equal(read_cache(ctx, b1), apply(c0, rows(1), 4))
    np.testing.assert_array_equal(read_cache(ctx, b0), c0)
    core.destroy_buffer(ctx, b1)
    core.destroy_buffer(ctx, b0)
