"""Host-side checks of the computed attention mask (no device needed).

generate-causal-mask (attention.clj:189-224) prints the additive mask either
as an iota / compare / select chain over the traced position or, for a
numeric position, as a dense literal.  The planner proves either form equal to
``mv where j - qpos > gt or j - qpos < lt, else z`` and the attention kernels
compute it instead of reading it.  These tests plan the printed graphs of the
three families and check the proven parameters against the reference's
semantics (masked when j > p + i, or j < p + i - window on local layers), and
that a literal that is not of the form stays a read mask.
"""
import dataclasses
import os
import re
import subprocess
import sys

import pytest

from cljxla_b200.host import core, drivers as d
from cljxla_b200.host import stablehlo as shlo

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAMILIES = {
    "gpt2": dataclasses.replace(d.GPT2_SMALL, vocab=96, d_model=384, layers=2, n_heads=12, n_kv_heads=12,
                                head_dim=32, mlp=128, n_positions=64),
    "gemma2": dataclasses.replace(d.GEMMA2_2B, vocab=64, d_model=64, layers=2, n_heads=4, n_kv_heads=2,
                                  head_dim=64, mlp=64, window=6),
    "gemma3": dataclasses.replace(d.GEMMA3_4B, vocab=64, d_model=64, layers=6, n_heads=4, n_kv_heads=2,
                                  head_dim=64, mlp=64, window=6),
}
FORMS = [("decode", False), ("prefill", False), ("prefill", True)]
LINE = re.compile(r"computed mask gt (-?\d+) lt (none )?(-?\d+) off (-?\d+) mv (\S+) z (\S+) pos (\S+)")


@pytest.fixture(scope="module")
def lib_path():
    import __graft_entry__
    __graft_entry__.build()
    from cljxla_b200 import LIB_PATH
    return LIB_PATH


def _plan_forms(lib_path, text, env_extra=None):
    """Plans `text` in a child process with the attention debug print on;
    returns (plan info, [(gt, lt or None, off, mv, z, pos name)])."""
    env = dict(os.environ, CLJXLA_B200_DEBUG_ATTN="1", **(env_extra or {}))
    code = ("import sys, json; sys.path.insert(0, %r); import __graft_entry__ as g; g._pkg();"
            "from cljxla_b200.host import core; t = sys.stdin.read();"
            "print(json.dumps(core.plan_text(%r, t)))" % (ROOT, lib_path))
    r = subprocess.run([sys.executable, "-c", code], input=text, capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    import json
    info = json.loads(r.stdout.strip().splitlines()[-1])
    forms = []
    for m in LINE.finditer(r.stderr):
        forms.append((int(m.group(1)), None if m.group(2) else int(m.group(3)), int(m.group(4)),
                      float(m.group(5)), float(m.group(6)), m.group(7)))
    return info, forms


@pytest.mark.parametrize("family", sorted(FAMILIES))
@pytest.mark.parametrize("kind,dynamic", FORMS)
def test_printed_masks_are_computed(lib_path, family, kind, dynamic):
    cfg = FAMILIES[family]
    S = 12 if kind == "prefill" else 1
    text = shlo.graph_to_mlir_text(d.build_graph(cfg, kind, 1, 12, 32, dynamic_prefill=dynamic))
    info, forms = _plan_forms(lib_path, text)
    assert info["computed_masks"] == cfg.layers == len(forms)
    for i, (gt, lt, off, mv, z, pos) in enumerate(forms):   # planned in layer order
        assert (gt, off, mv, z) == (0, 0, -10000.0, 0.0)
        window = cfg.window if cfg.is_local(i) else None
        # a static prefill literal spans only S positions: a window >= S - 1 masks nothing there
        if window is not None and kind == "prefill" and not dynamic and window >= S - 1:
            window = None
        assert lt == (None if window is None else -window), (i, lt)
        static = kind == "prefill" and not dynamic
        assert (pos == "-") == static, pos


def test_switch_keeps_read_masks(lib_path):
    text = shlo.graph_to_mlir_text(d.build_graph(FAMILIES["gemma3"], "decode", 1, 12, 32))
    on = core.plan_text(lib_path, text)
    info, forms = _plan_forms(lib_path, text, {"CLJXLA_B200_MASK_FORM": "0"})
    assert info["computed_masks"] == 0 and not forms
    # the mask chain is no longer computed by its own kernel
    assert on["launches"] < info["launches"] and on["live_nodes"] < info["live_nodes"]


def _decode_text():
    return shlo.graph_to_mlir_text(d.build_graph(FAMILIES["gemma3"], "decode", 1, 12, 32))


def _first(text, old, new):
    assert old in text, old
    return text.replace(old, new, 1)


@pytest.mark.parametrize("mutation,layer0", [
    # an equivalent window test: d <= -7 is d < -6
    ("le", (0, -6)),
    # another window: the proof reads the threshold, it does not assume it
    ("window5", (0, -5)),
    # d >= 0 also masks the query's own position: gt -1
    ("ge", (-1, -6)),
], ids=["le-is-lt", "other-window", "ge-masks-diagonal"])
def test_mask_chain_variants_are_read_exactly(lib_path, mutation, layer0):
    """Edits of layer 0's printed mask chain that keep it of the closed form are
    proven with the thresholds they mean (the other layers keep theirs)."""
    text = _decode_text()
    if mutation == "le":
        text = _first(text, "dense<[-6.000000e+00]>", "dense<[-7.000000e+00]>")
        text = _first(text, "comparison_direction LT>", "comparison_direction LE>")
    elif mutation == "window5":
        text = _first(text, "dense<[-6.000000e+00]>", "dense<[-5.000000e+00]>")
    else:
        text = _first(text, "comparison_direction GT>", "comparison_direction GE>")
    info, forms = _plan_forms(lib_path, text)
    assert info["computed_masks"] == FAMILIES["gemma3"].layers == len(forms)
    assert (forms[0][0], forms[0][1]) == layer0
    assert all((f[0], f[1]) == (0, -6) for f in forms[1:5]) and forms[5][:2] == (0, None)


def test_mask_chain_not_of_the_form_stays_read(lib_path):
    """Layer 0's compared value turned around (i + p - j: an anti-causal mask)
    and layer 1's position taken twice (j - i - 2p) are not the closed form:
    those layers read their masks, the others stay computed."""
    text = _decode_text()
    m = re.search(r"stablehlo\.subtract %(\S+), %(\S+) : tensor<1x1x1x32xf32>", text)
    text = text[:m.start()] + f"stablehlo.subtract %{m.group(2)}, %{m.group(1)} : tensor<1x1x1x32xf32>" + \
        text[m.end():]
    # layer 1: its i + p add becomes i + p + p (the position reshaped once more)
    adds = list(re.finditer(r"%(t_add_\d+) = stablehlo\.add %(\S+), %(\S+) : tensor<1x1x1x1xf32>", text))
    a = adds[1]
    text = text[:a.start()] + (f"%{a.group(1)}_p = stablehlo.add %{a.group(2)}, %{a.group(3)} : tensor<1x1x1x1xf32>\n"
                               f"    %{a.group(1)} = stablehlo.add %{a.group(1)}_p, %{a.group(3)} : "
                               f"tensor<1x1x1x1xf32>") + text[a.end():]
    info, forms = _plan_forms(lib_path, text)
    assert info["computed_masks"] == FAMILIES["gemma3"].layers - 2 == len(forms)


def test_literal_not_of_the_form_stays_read(lib_path):
    cfg = FAMILIES["gemma3"]
    text = shlo.graph_to_mlir_text(d.build_graph(cfg, "prefill", 1, 12, 32))
    lit = re.search(r"constant dense<\[([^\]]*)\]> : tensor<144xf32>", text)
    assert lit, "the static prefill prints its 12 x 12 mask as a flat literal"
    vals = lit.group(1).split(", ")
    assert vals[1] == "-1.000000e+04"
    vals[1] = "0.000000e+00"            # query 0 now sees position 1 too: not causal
    bad = text[:lit.start(1)] + ", ".join(vals) + text[lit.end(1):]
    info, forms = _plan_forms(lib_path, bad)
    good, _ = _plan_forms(lib_path, text)
    assert good["computed_masks"] == cfg.layers
    assert info["computed_masks"] < cfg.layers
    assert info["const_bytes"] > good["const_bytes"]    # the odd literal is uploaded and read
