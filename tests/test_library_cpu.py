"""Host-side checks of libcljxla_b200.so (no device needed): the library loads,
exports every symbol include/*.h declares, and parses + plans the decoder
graphs of every BASELINE architecture; malformed / unsupported programs come
back as PJRT error codes, never aborts."""
import ctypes
import dataclasses
import os
import re

import pytest

from cljxla_b200.host import core, drivers as d
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200.host import tensor as t

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib_path():
    import __graft_entry__
    __graft_entry__.build()
    from cljxla_b200 import LIB_PATH
    return LIB_PATH


def declared_symbols():
    syms = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        txt = open(os.path.join(ROOT, "include", h)).read()
        for m in re.finditer(r"CLJXLA_EXPORT\s+[\w\s\*]+?\b(\w+)\s*\(", txt):
            syms.add(m.group(1))
    return syms


def test_library_exports_declared_symbols(lib_path):
    lib = ctypes.CDLL(lib_path)
    syms = declared_symbols()
    assert "GetPjrtApi" in syms
    for s in syms:
        assert hasattr(lib, s), s


def test_pjrt_table_layout(lib_path):
    from cljxla_b200.host.pjrt import PjrtApi, OFFSET_LOADED_EXECUTABLE_EXECUTE, _r64
    lib = ctypes.CDLL(lib_path)
    lib.GetPjrtApi.restype = ctypes.c_void_p
    p = lib.GetPjrtApi()
    api = (ctypes.c_char * 984).from_address(p)
    assert _r64(api, 0) == 984
    for off in range(40, 984, 8):  # every slot is callable (real entry or UNIMPLEMENTED stub)
        assert _r64(api, off) != 0
    # plugin initialize works without a device
    ap = PjrtApi(lib_path)
    assert ap.plugin_attributes()["stablehlo_current_version"] == "1.0.0"


@pytest.mark.parametrize("name", ["gpt2-small", "gemma2-2b", "gemma3-4b", "gemma3-12b", "gemma3-27b"])
def test_plan_full_size_decode_graphs(lib_path, name):
    cfg = d.CONFIGS[name]
    S = {"gpt2-small": 128, "gemma2-2b": 512, "gemma3-4b": 2048, "gemma3-12b": 4096, "gemma3-27b": 8192}[name]
    T = d.round_up(S + 256, 128)
    txt = shlo.graph_to_mlir_text(d.build_graph(cfg, "decode", 1, S, T))
    info = core.plan_text(lib_path, txt)
    assert info["launches"] > 0 and info["live_nodes"] < info["nodes"] + 1


@pytest.mark.parametrize("family", ["gpt2-small", "gemma2-2b", "gemma3-4b"])
def test_plan_prefill_graphs(lib_path, family):
    cfg = d.CONFIGS[family]
    cfg = dataclasses.replace(cfg, layers=2)
    for dyn in (False, True):
        txt = shlo.graph_to_mlir_text(d.build_graph(cfg, "prefill", 1, 64, 128, dynamic_prefill=dyn))
        assert core.plan_text(lib_path, txt)["launches"] > 0


def test_parse_errors_have_codes(lib_path):
    with pytest.raises(RuntimeError, match=r"\(3\)"):
        core.plan_text(lib_path, "module @x {\n  nonsense\n}\n")
    bad_op = ("module @x {\n  func.func @main(%a: tensor<2xf32>) -> (tensor<2xf32>) {\n"
              "    %b = stablehlo.cbrt %a : tensor<2xf32>\n    return %b : tensor<2xf32>\n  }\n}\n")
    with pytest.raises(RuntimeError, match=r"\(12\)"):
        core.plan_text(lib_path, bad_op)
    undefined = ("module @x {\n  func.func @main(%a: tensor<2xf32>) -> (tensor<2xf32>) {\n"
                 "    %b = stablehlo.add %a, %zz : tensor<2xf32>\n    return %b : tensor<2xf32>\n  }\n}\n")
    with pytest.raises(RuntimeError, match=r"undefined value"):
        core.plan_text(lib_path, undefined)


def test_loc_suffix_is_ignored(lib_path):
    g = t.trace_graph("m", [("x", ("tensor", (2, 3), "f32"))], lambda x: t.tanh(x))
    g["eqns"][-1]["metadata"] = {"op-name": "layer0/act"}
    txt = shlo.graph_to_mlir_text(g)
    assert 'loc("layer0/act")' in txt
    assert core.plan_text(lib_path, txt)["launches"] >= 1


def test_debug_checks_are_dropped_with_dead_code(lib_path):
    """debug.clj's check-non-nan / check-non-inf print as custom_call ops
    whose tensor<i1> result nothing uses (stablehlo.clj:562-570): a model graph
    carrying them (with their loc suffix) plans to the same launches as without
    them.  A check whose result the graph returns, or any other custom_call
    target, is UNIMPLEMENTED."""
    cfg = dataclasses.replace(d.GEMMA3_4B, vocab=64, d_model=64, layers=2, n_heads=4, n_kv_heads=2,
                              head_dim=64, mlp=64, window=6)
    txt = shlo.graph_to_mlir_text(d.build_graph(cfg, "decode", 1, 12, 32))
    base = core.plan_text(lib_path, txt)
    m = re.search(r"\n(\s*)%(t_\w+) = stablehlo\.multiply %\S+, %\S+ : (tensor<[^>]*xf32>)\n", txt)
    ind, v, ty = m.group(1), m.group(2), m.group(3)
    checks = (f'{ind}%chk_nan_1 = "stablehlo.custom_call"(%{v}) {{call_target_name = "check_non_nan"}} : '
              f'({ty}) -> tensor<i1> loc("gemma/layer_0/check")\n'
              f'{ind}%chk_inf_2 = "stablehlo.custom_call"(%{v}) {{call_target_name = "check_non_inf"}} : '
              f'({ty}) -> tensor<i1>\n')
    with_checks = txt[:m.end()] + checks + txt[m.end():]
    got = core.plan_text(lib_path, with_checks)
    assert got["launches"] == base["launches"] and got["live_nodes"] == base["live_nodes"]
    # the oracle evaluates the checks and computes the same results
    import numpy as np
    from oracle import interp
    ins = [d.make_prompt(cfg, 1, 1), d.pos_inputs(cfg, "decode", 1, 12, 1)] + d.make_weights(cfg) + \
        [d.zero_cache(cfg, 1, 32) for _ in range(2 * cfg.layers)]
    a, b = interp.run_mlir(txt, ins), interp.run_mlir(with_checks, ins)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    # the first result (the logits) replaced by the check
    returned = re.sub(r"return %\w+, (.*) : tensor<[^>]*>, ", r"return %chk_nan_1, \1 : tensor<i1>, ", with_checks, 1)
    returned = re.sub(r"\) -> \(tensor<[^>]*>, ", ") -> (tensor<i1>, ", returned, 1)
    assert returned.count("tensor<i1>, ") >= 2
    with pytest.raises(RuntimeError, match=r"\(12\).*check_non_nan"):
        core.plan_text(lib_path, returned)
    other = with_checks.replace('"check_non_inf"', '"embed_lookup"')
    with pytest.raises(RuntimeError, match=r"\(12\).*embed_lookup"):
        core.plan_text(lib_path, other)


def test_generated_fused_kernels_compile(lib_path):
    """Every fused elementwise / row kernel the planner generates for the
    model graphs compiles with NVRTC for sm_100a (host only)."""
    import ctypes
    import dataclasses
    from cljxla_b200.host import drivers as d
    from cljxla_b200.host import stablehlo as shlo
    lib = ctypes.CDLL(lib_path)
    f = lib.cljxla_b200_jit_check
    f.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p,
                  ctypes.c_size_t]
    f.restype = ctypes.c_int
    tiny = {
        "gpt2": dataclasses.replace(d.GPT2_SMALL, vocab=384, d_model=384, layers=2, n_heads=12, n_kv_heads=12,
                                    head_dim=32, mlp=768, n_positions=64),
        "gemma2": dataclasses.replace(d.GEMMA2_2B, vocab=512, d_model=256, layers=2, n_heads=4, n_kv_heads=2,
                                      head_dim=64, mlp=512, window=6),
        "gemma3": dataclasses.replace(d.GEMMA3_4B, vocab=512, d_model=256, layers=6, n_heads=4, n_kv_heads=2,
                                      head_dim=64, mlp=512, window=6),
    }
    for name, cfg in tiny.items():
        for kind in ("prefill", "decode"):
            text = shlo.graph_to_mlir_text(d.build_graph(cfg, kind, 1, 8, 16, dynamic_prefill=kind == "prefill"))
            b = text.encode()
            k = ctypes.c_int(0)
            err = ctypes.create_string_buffer(1 << 16)
            rc = f(b, len(b), 3, ctypes.byref(k), err, 1 << 16)
            if rc == -1:
                pytest.skip("NVRTC not available")
            assert rc == 0, f"{name} {kind}: {rc} of {k.value} kernels failed\n{err.value.decode()[:4000]}"
            assert k.value > 0


def test_decode_plan_fusions(lib_path, monkeypatch):
    """The decode plan's launch count with and without each fusion (host-only
    planning): the GeGLU runs as the gate / up GEMV's epilogue, RoPE in the
    CTAs of the per-head norms, and single-row norms as GEMV prologues; every
    fused kernel still has its compiled form (checked in
    test_generated_fused_kernels_compile)."""
    import dataclasses
    from cljxla_b200.host import drivers as d
    from cljxla_b200.host import stablehlo as shlo
    cfg = dataclasses.replace(d.GEMMA3_4B, vocab=512, d_model=256, layers=6, n_heads=4, n_kv_heads=2,
                              head_dim=64, mlp=512, window=6)
    text = shlo.graph_to_mlir_text(d.build_graph(cfg, "decode", 1, 8, 32))

    def launches(**env):
        for k in ("CLJXLA_B200_GEMV_EPILOGUE", "CLJXLA_B200_ROW_EPILOGUE", "CLJXLA_B200_GEMV_PROLOGUE"):
            monkeypatch.delenv(k, raising=False)
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        return core.plan_text(lib_path, text, fuse=3)["launches"]

    full = launches()
    assert launches(CLJXLA_B200_GEMV_EPILOGUE="0") >= full + cfg.layers
    assert launches(CLJXLA_B200_ROW_EPILOGUE="0") >= full + cfg.layers
    assert launches(CLJXLA_B200_GEMV_PROLOGUE="0") >= full + cfg.layers
    # six launches per layer: attention, o, gate/up (+ norm prologue, GeGLU epilogue), down,
    # q/k/v (+ input norm prologue), per-head norms (+ RoPE and the KV writes)
    assert full <= 6 * cfg.layers + 8, full


_JIT_CACHE_PROBE = r"""
import ctypes, sys, dataclasses
sys.path.insert(0, sys.argv[1])
import conftest
from cljxla_b200.host import drivers as d
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200 import LIB_PATH
lib = ctypes.CDLL(LIB_PATH)
cfg = dataclasses.replace(d.GEMMA3_4B, vocab=512, d_model=256, layers=2, n_heads=4, n_kv_heads=2,
                          head_dim=64, mlp=512, window=6)
b = shlo.graph_to_mlir_text(d.build_graph(cfg, "decode", 1, 8, 16)).encode()
f = lib.cljxla_b200_jit_check
f.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p,
              ctypes.c_size_t]
k = ctypes.c_int(0)
rc = f(b, len(b), 3, ctypes.byref(k), None, 0)
hits, misses = ctypes.c_int64(0), ctypes.c_int64(0)
lib.cljxla_b200_jit_cache_stats(ctypes.byref(hits), ctypes.byref(misses))
print(rc, k.value, hits.value, misses.value)
"""


def test_compiled_kernels_persist_across_processes(lib_path, tmp_path):
    """A second process compiling the same graph takes every fused kernel from
    the on-disk cache (SHA-256 keyed, like clj-xla's compile cache) instead of
    running NVRTC again; with the cache turned off nothing is written."""
    import subprocess
    import sys
    env = dict(os.environ, CLJXLA_B200_CACHE_DIR=str(tmp_path / "cache"))
    probe = [sys.executable, "-c", _JIT_CACHE_PROBE, os.path.join(ROOT, "tests")]
    first = subprocess.run(probe, env=env, capture_output=True, text=True, cwd=ROOT)
    rc, kernels, hits, misses = map(int, first.stdout.split()[-4:])
    if rc == -1:
        pytest.skip("NVRTC not available")
    assert rc == 0 and kernels > 0 and hits == 0 and misses > 0, first.stdout + first.stderr
    files = sorted(p.name for p in (tmp_path / "cache").iterdir())
    assert len(files) == misses and all(re.fullmatch(r"[0-9a-f]{64}\.cubin", n) for n in files), files
    second = subprocess.run(probe, env=env, capture_output=True, text=True, cwd=ROOT)
    rc2, kernels2, hits2, misses2 = map(int, second.stdout.split()[-4:])
    assert (rc2, kernels2, hits2, misses2) == (0, kernels, misses, 0), second.stdout + second.stderr
    off = subprocess.run(probe, env=dict(os.environ, CLJXLA_B200_CACHE_DIR="0"), capture_output=True, text=True,
                         cwd=ROOT)
    assert list(map(int, off.stdout.split()[-4:]))[2:] == [0, 0], off.stdout + off.stderr
