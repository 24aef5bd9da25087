"""Golden MLIR text for the reference's own example graphs.

Expected strings are derived by hand from the printer rules in
src/clj_xla/stablehlo.clj (scalar constants print as ``tensor<f32>`` with a
``broadcast_in_dim`` inserted at the use, :254-270 and :515-518) for the graphs
in README.md:50-55, test/clj_xla/pjrt_test.clj:37-41,
test/clj_xla/compile_test.clj:12-16 and
test/clj_xla/integration/rocm_e2e_test.clj:28-46.
"""
from cljxla_b200.host import stablehlo as shlo
from cljxla_b200.host import tensor as t


def _mul_graph(name, shape, c):
    return {"name": name, "invars": [("x", ("tensor", shape, "f32"))], "outvars": ["y"],
            "eqns": [{"op": "stablehlo/constant", "value": c, "outvars": ["c0"]},
                     {"op": "stablehlo/multiply", "invars": ["x", "c0"], "outvars": ["y"]}]}


def _expected_mul(name, tstr, cstr):
    return (f"module @{name} {{\n"
            f"  func.func @main(%x: {tstr}) -> ({tstr}) {{\n"
            f"    %c0 = stablehlo.constant dense<{cstr}> : tensor<f32>\n"
            f'    %c0_bcast_y = "stablehlo.broadcast_in_dim"(%c0) {{broadcast_dimensions = array<i64>}} : (tensor<f32>) -> {tstr}\n'
            f"    %y = stablehlo.multiply %x, %c0_bcast_y : {tstr}\n"
            f"    return %y : {tstr}\n"
            "  }\n"
            "}\n")


def test_readme_gelu_block_golden():
    g = _mul_graph("gelu_block", (1, 128, 768), 0.5)
    assert shlo.graph_to_mlir_text(g) == _expected_mul("gelu_block", "tensor<1x128x768xf32>", "5.000000e-01")


def test_pjrt_compile_module_golden():
    g = _mul_graph("test_compile_module", (1, 64), 1.5)
    assert shlo.graph_to_mlir_text(g) == _expected_mul("test_compile_module", "tensor<1x64xf32>", "1.500000e+00")


def test_compile_cache_graph_golden():
    g = _mul_graph("cached_graph", (2, 32), 3.0)
    assert shlo.graph_to_mlir_text(g) == _expected_mul("cached_graph", "tensor<2x32xf32>", "3.000000e+00")


def test_rocm_parity_graph_golden():
    g = _mul_graph("parity_test_graph", (1, 16), 2.5)
    assert shlo.graph_to_mlir_text(g) == _expected_mul("parity_test_graph", "tensor<1x16xf32>", "2.500000e+00")


def test_rocm_two_input_graph_golden():
    g = {"name": "rocm_compile", "invars": [("x", ("tensor", (1, 64), "f32")), ("y", ("tensor", (1, 64), "f32"))],
         "outvars": ["z"], "eqns": [{"op": "stablehlo/multiply", "invars": ["x", "y"], "outvars": ["z"]}]}
    assert shlo.graph_to_mlir_text(g) == (
        "module @rocm_compile {\n"
        "  func.func @main(%x: tensor<1x64xf32>, %y: tensor<1x64xf32>) -> (tensor<1x64xf32>) {\n"
        "    %z = stablehlo.multiply %x, %y : tensor<1x64xf32>\n"
        "    return %z : tensor<1x64xf32>\n"
        "  }\n"
        "}\n")


def test_type_to_mlir_string_cases():
    # stablehlo_test.clj:56-60
    assert shlo.type_to_mlir(("tensor", (1, 128, 768), "f32")) == "tensor<1x128x768xf32>"
    assert shlo.type_to_mlir(("tensor", (10,), "f16")) == "tensor<10xf16>"
    assert shlo.type_to_mlir(("tensor", (), "f32")) == "tensor<f32>"


def test_invalid_graph_rejected():
    import pytest
    with pytest.raises(ValueError):
        t.validate_graph({"invalid": True})
    with pytest.raises(ValueError):
        t.validate_graph({"name": "bad", "invars": [], "outvars": [], "eqns": "not-a-vector"})


def test_traced_scalar_rhs_inherits_type_and_lhs_scalar_broadcasts():
    # tensor.clj:55-80: (* x 2.0) -> constant of x's full type; (* 2.0 x) -> f32 scalar + broadcast,
    # then the printer re-infers the result as x's type and inserts a convert (stablehlo.clj:499-510)
    g = t.trace_graph("m", [("x", ("tensor", (2, 3), "bf16"))], lambda x: t.mul(2.0, t.mul(x, 2.0)))
    txt = shlo.graph_to_mlir_text(g)
    assert "%c_1 = stablehlo.constant dense<2.000000e+00> : tensor<2x3xbf16>" in txt
    assert "%c_3 = stablehlo.constant dense<2.000000e+00> : tensor<f32>" in txt
    assert '"stablehlo.broadcast_in_dim"(%c_3) {broadcast_dimensions = array<i64>} : (tensor<f32>) -> tensor<2x3xf32>' in txt
    assert '%t_bcast_4_conv_t_mul_5 = "stablehlo.convert"(%t_bcast_4) : (tensor<2x3xf32>) -> tensor<2x3xbf16>' in txt
    assert "%t_mul_5 = stablehlo.multiply %t_bcast_4_conv_t_mul_5, %t_mul_2 : tensor<2x3xbf16>" in txt


def test_reduce_prints_region_and_init():
    g = t.trace_graph("r", [("x", ("tensor", (2, 8), "f32"))], lambda x: t.reduce_max(x))
    txt = shlo.graph_to_mlir_text(g)
    assert "%t_max_1_c0 = stablehlo.constant dense<-1.000000e+30> : tensor<f32>" in txt
    assert "{dimensions = array<i64: 1>} : (tensor<2x8xf32>, tensor<f32>) -> tensor<2xf32>" in txt
    assert "%t_max_1 = stablehlo.reshape %t_max_1_red : (tensor<2xf32>) -> tensor<2x1xf32>" in txt
