"""cljxla_b200_attention_decode_static: decode attention without allocation.

The entry point runs the split-KV attention kernels with their partials in a
fixed device array.  It is compared with the existing entry point - the same
attention block printed as a graph (attention.clj:343-365) and run through
PJRT Execute, where the planner matches it to the same kernels with the
partials in the executable's scratch - within the f32 tolerance the other
parity tests use, on two calls in a row, for a split case (partials in the
array), a Gemma-3 sliding-window layer at head_dim 256 and a one-split case.
The second call must leave the device's free memory and the default memory
pool's reserved and used bytes unchanged.
"""
import ctypes

import numpy as np
import pytest

from cljxla_b200.host import core
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200.host import tensor as t
from cljxla_b200.host.pjrt import DTYPE_ENUM
from oracle import interp

from conftest import has_gpu
from parity import close

pytestmark = pytest.mark.gpu

# (batch, q heads, kv heads, positions, head_dim, scale, first masked position, window)
CASES = {
    # 8 splits of 80 positions: partials in the static array, merged by the combine kernel
    "hd128_causal": (2, 8, 4, 640, 128, 0.0625, 500, None),
    # a Gemma-3 local layer at decode position 2047: 1024-position window, head_dim 256
    "hd256_window": (1, 8, 4, 2560, 256, 1.0, 2048, 1024),
    # 96 positions: one split, no partials and no combine
    "hd64_one_split": (1, 4, 2, 96, 64, 0.125, 90, None),
}


@pytest.fixture(scope="module")
def ctx():
    if not has_gpu():
        pytest.skip("no CUDA device")
    from cljxla_b200 import LIB_PATH
    return core.init_backend(LIB_PATH)


def attention_graph(case):
    B, NQ, NKV, T, HD, SCALE, _, _ = case
    g = NQ // NKV

    def f(q, kc, vc, mask):
        kh = t.reshape(t.broadcast_in_dim(kc, [B, NKV, g, T, HD], [0, 1, 3, 4]), [B, NQ, T, HD])
        vh = t.reshape(t.broadcast_in_dim(vc, [B, NKV, g, T, HD], [0, 1, 3, 4]), [B, NQ, T, HD])
        raw = t.dot_general(q, kh, {"batch_dims": {"lhs": [0, 1], "rhs": [0, 1]},
                                    "contracting_dims": {"lhs": [3], "rhs": [3]}})
        masked = t.add(t.mul(raw, SCALE), mask)
        ex = t.exp(t.sub(masked, t.reduce_max(masked, axes=[-1], keep_dims=True)))
        probs = t.div(ex, t.reduce_sum(ex, axes=[-1], keep_dims=True))
        return [t.dot_general(probs, vh, {"batch_dims": {"lhs": [0, 1], "rhs": [0, 1]},
                                          "contracting_dims": {"lhs": [3], "rhs": [2]}})]

    return t.trace_graph("attn_static", [("q", ("tensor", (B, NQ, 1, HD), "bf16")),
                                         ("kc", ("tensor", (B, NKV, T, HD), "bf16")),
                                         ("vc", ("tensor", (B, NKV, T, HD), "bf16")),
                                         ("mask", ("tensor", (1, 1, 1, T), "f32"))], f)


def inputs(case):
    B, NQ, NKV, T, HD, _, first_masked, window = case
    rng = np.random.Generator(np.random.PCG64(11))
    bf = lambda shape: interp.f32_to_bf16_bits(rng.standard_normal(shape).astype(np.float32))
    mask = np.zeros((1, 1, 1, T), np.float32)
    mask[..., first_masked:] = -10000.0  # positions past the current one
    if window is not None:              # positions more than `window` behind the current one
        mask[..., :max(0, first_masked - 1 - window)] = -10000.0
    return [bf((B, NQ, 1, HD)), bf((B, NKV, T, HD)), bf((B, NKV, T, HD)), mask]


def static_fn(lib):
    f = lib.cljxla_b200_attention_decode_static
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 5 + [ctypes.c_float, ctypes.c_void_p,
                                                                  ctypes.c_char_p, ctypes.c_size_t]
    f.restype = ctypes.c_int
    return f


def dev_ptr(lib, buf):
    f = lib.cljxla_b200_buffer_device_pointer
    f.argtypes = [ctypes.c_void_p]
    f.restype = ctypes.c_void_p
    return f(ctypes.c_void_p(buf))


def _cudart():
    """The CUDA runtime torch loaded, for the device memory-pool counters."""
    import torch
    torch.cuda.init()
    for line in open("/proc/self/maps"):
        path = line.split()[-1] if line.rstrip().endswith(".so") or ".so." in line else ""
        if "libcudart.so" in path:
            return ctypes.CDLL(path)
    return None


def _memory_state(rt):
    """(free device bytes, default-pool reserved bytes, default-pool used bytes)."""
    import torch
    free, _ = torch.cuda.mem_get_info()
    if rt is None:
        return free, None, None
    pool = ctypes.c_void_p()
    assert rt.cudaDeviceGetDefaultMemPool(ctypes.byref(pool), torch.cuda.current_device()) == 0
    vals = []
    for attr in (5, 7):  # cudaMemPoolAttrReservedMemCurrent, cudaMemPoolAttrUsedMemCurrent
        v = ctypes.c_uint64()
        assert rt.cudaMemPoolGetAttribute(pool, attr, ctypes.byref(v)) == 0
        vals.append(v.value)
    return (free, *vals)


@pytest.mark.parametrize("name", list(CASES))
def test_static_scratch_matches_execute_twice(ctx, name):
    case = CASES[name]
    B, NQ, NKV, T, HD, SCALE = case[:6]
    g = attention_graph(case)
    text = shlo.graph_to_mlir_text(g)
    exe = core.compile_mlir_text(ctx, text, g)
    assert core.plan_info(ctx, exe)["launches"] == 1  # matched: attention, splits merged in-kernel
    host = inputs(case)
    api, lib = ctx["api"], ctx["api"].lib
    bufs = [core.buffer_from_host_buffer(ctx, a, a.shape, DTYPE_ENUM[dt])
            for a, dt in zip(host, ["bf16", "bf16", "bf16", "f32"])]
    out_buf = core.buffer_from_host_buffer(ctx, np.zeros((B, NQ, 1, HD), np.float32), (B, NQ, 1, HD), DTYPE_ENUM["f32"])
    try:
        ref_buf = api.execute_executable(exe["handle"], bufs, 1)
        ref_buf = ref_buf[0] if isinstance(ref_buf, list) else ref_buf
        want = core.buffer_to_numpy(ctx, ref_buf, (B, NQ, 1, HD), "f32")
        core.destroy_buffer(ctx, ref_buf)
        oracle = interp.run_mlir(text, host)[0]
        assert close(want, oracle, "f32")[0]
        fn = static_fn(lib)
        ptrs = [dev_ptr(lib, b) for b in bufs] + [dev_ptr(lib, out_buf)]
        err = ctypes.create_string_buffer(512)
        rt = _cudart()
        stream = core.client_stream(ctx)
        for call in range(2):
            before = _memory_state(rt)
            rc = fn(*[ctypes.c_void_p(p) for p in ptrs], B, NQ, NKV, T, HD, SCALE,
                    ctypes.c_void_p(stream), err, 512)
            after = _memory_state(rt)
            assert rc == 0, err.value.decode()
            got = core.buffer_to_numpy(ctx, out_buf, (B, NQ, 1, HD), "f32")
            ok, excess, maxerr = close(got, want, "f32")
            assert ok, f"call {call}: max err {maxerr:.3g}, excess {excess:.3g}"
            if call == 1:  # the first call may load the module; the second must take no memory at all
                assert after == before, f"device memory changed across a call: {before} -> {after}"
    finally:
        for b in bufs + [out_buf]:
            core.destroy_buffer(ctx, b)


def test_static_scratch_rejects_oversized_requests(ctx):
    lib = ctx["api"].lib
    fn = static_fn(lib)
    err = ctypes.create_string_buffer(512)
    # one KV head over 65536 positions takes 256 splits: 256 x 8 heads x 258 floats > 1 MiB,
    # refused on the host before anything is launched
    one = ctypes.c_void_p(16)
    rc = fn(one, one, one, one, one, 1, 8, 1, 65536, 256, 1.0, None, err, 512)
    assert rc == 3 and b"static scratch" in err.value
    rc = fn(one, one, one, one, one, 1, 8, 4, 64, 96, 1.0, None, err, 512)
    assert rc == 3 and b"head_dim" in err.value
