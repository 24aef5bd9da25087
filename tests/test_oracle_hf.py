"""Pins the oracle at model level against an independent implementation of the
three architectures: the Hugging Face ``transformers`` models, which the
reference's own verification scripts use as their anchor
(verification/verify_torch_vs_clojure.py, verification/test_hf_transformers.py).

Each case traces the reference's graph with the host mirror (f32, tiny sizes),
runs a dynamic-position prefill and three cached decode steps through
``oracle/interp.py``, and compares every position's logits with one HF forward
over the whole sequence, on the same weights.  Known, deliberate differences
between the reference's graphs and HF's modules are mapped, each from the
reference file that defines it:

* sliding window: the reference masks key j of query position p only when
  ``j < p - window`` (nn/attention.clj:212-224), so a window of W admits W + 1
  keys; HF's ``sliding_window`` counts the query's own position, hence W + 1;
* Gemma-3 (a block with QK-norm): norms are plain ``x * w`` (gemma.clj:146-147,
  nn/norm.clj ``rms-norm``) where HF stores ``w - 1`` for ``x * (1 + w)``; V is
  RMS-normalised over the whole kv_dim without a weight (gemma.clj:167); the
  attention scale is 1.0 (gemma.clj:179), i.e. HF's query_pre_attn_scalar 1;
  global layers use RoPE base 1e6, local ones 1e4 (the 5:1 pattern);
* GPT-2: GELU is the tanh form (nn/activations.clj:7-11, HF ``gelu_new``),
  LayerNorm eps 1e-5, tied LM head.

Tolerance: parity.clj:36-49's ``approx-equal?`` at atol = rtol = 1e-4 on f32.
"""
import dataclasses

import numpy as np
import pytest

from cljxla_b200.host import drivers as d
from cljxla_b200.host import stablehlo as shlo
from oracle import interp

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")

S, T, DECODE = 10, 16, 3
BATCHES = [1, 2]   # batch 2: the batched gather, attention and cache layout of the graphs


def approx_equal(a, b, atol=1e-4, rtol=1e-4):
    """parity.clj:36-49 ``approx-equal?``."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return a.shape == b.shape and bool(np.all(np.abs(a - b) <= atol + rtol * np.abs(b)))


def oracle_logits(cfg, w, toks):
    """Prefill of the first S tokens, then DECODE single-token steps on the
    returned caches: logits of every position, [B, S + DECODE, V]."""
    B = toks.shape[0]
    g = d.build_graph(cfg, "prefill", B, S, T, dynamic_prefill=True)
    inputs = [toks[:, :S], d.pos_inputs(cfg, "prefill", B, 0, S)] + w + \
        [d.zero_cache(cfg, B, T) for _ in range(2 * cfg.layers)]
    out = interp.run_mlir(shlo.graph_to_mlir_text(g), inputs)
    logits = [np.asarray(out[0]).reshape(B, -1, cfg.vocab)]
    caches = out[1:]
    text = shlo.graph_to_mlir_text(d.build_graph(cfg, "decode", B, 1, T))
    for s in range(S, S + DECODE):
        o = interp.run_mlir(text, [toks[:, s:s + 1], d.pos_inputs(cfg, "decode", B, s, 1)] + w + list(caches))
        logits.append(np.asarray(o[0]).reshape(B, -1, cfg.vocab))
        caches = o[1:]
    return np.concatenate(logits, axis=1)


def hf_logits(model, sd, toks):
    sd = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert set(missing) <= {"lm_head.weight"}, missing   # tied to the embedding below
    model.tie_weights()
    model.lm_head.weight = model.get_input_embeddings().weight
    with torch.no_grad():
        return model(torch.from_numpy(toks).long()).logits.numpy()


@pytest.mark.parametrize("B", BATCHES)
def test_gpt2_matches_hf(B):
    from transformers import GPT2Config, GPT2LMHeadModel
    # gpt2.clj's block passes 12 heads
    cfg = dataclasses.replace(d.GPT2_SMALL, vocab=96, d_model=96, layers=2, n_heads=12, n_kv_heads=12,
                              head_dim=8, mlp=256, n_positions=32)
    w = d.make_weights(cfg)
    rng = np.random.default_rng(5)   # non-trivial LayerNorm and bias vectors
    w = [a + rng.standard_normal(a.shape).astype(np.float32) * np.float32(0.05) if a.ndim == 1 else a for a in w]
    W = dict(zip([n for n, _, _ in d.weight_specs(cfg)], w))
    toks = d.make_prompt(cfg, B, S + DECODE)
    hc = GPT2Config(vocab_size=cfg.vocab, n_positions=cfg.n_positions, n_embd=cfg.d_model, n_layer=cfg.layers,
                    n_head=cfg.n_heads, n_inner=cfg.mlp, activation_function="gelu_new",
                    layer_norm_epsilon=1e-5, attn_pdrop=0.0, resid_pdrop=0.0, embd_pdrop=0.0)
    sd = {"transformer.ln_f.weight": W["ln_f_g"], "transformer.ln_f.bias": W["ln_f_b"],
          "transformer.wte.weight": W["wte"], "transformer.wpe.weight": W["wpe"]}
    hf_name = {"ln1_g": "ln_1.weight", "ln1_b": "ln_1.bias", "attn_w": "attn.c_attn.weight",
               "attn_b": "attn.c_attn.bias", "proj_w": "attn.c_proj.weight", "proj_b": "attn.c_proj.bias",
               "ln2_g": "ln_2.weight", "ln2_b": "ln_2.bias", "mlp_fc_w": "mlp.c_fc.weight",
               "mlp_fc_b": "mlp.c_fc.bias", "mlp_proj_w": "mlp.c_proj.weight", "mlp_proj_b": "mlp.c_proj.bias"}
    for i in range(cfg.layers):
        for ours, theirs in hf_name.items():   # Conv1D weights are [in, out] on both sides
            sd[f"transformer.h.{i}.{theirs}"] = W[f"{ours}_{i}"]
    ref = hf_logits(GPT2LMHeadModel(hc).eval(), sd, toks)
    got = oracle_logits(cfg, w, toks)
    assert approx_equal(got, ref), float(np.abs(got - ref).max())


def _gemma_state(cfg, W):
    plain = cfg.family == "gemma3"
    norm = (lambda a: a - np.float32(1.0)) if plain else (lambda a: a)
    sd = {"model.embed_tokens.weight": W["embed_tokens"], "model.norm.weight": W["final_norm_w"]}
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        sd.update({p + "input_layernorm.weight": norm(W[f"input_ln_w_{i}"]),
                   p + "self_attn.q_proj.weight": W[f"q_w_{i}"], p + "self_attn.k_proj.weight": W[f"k_w_{i}"],
                   p + ("self_attn.v_proj.lin.weight" if plain else "self_attn.v_proj.weight"): W[f"v_w_{i}"],
                   p + "self_attn.o_proj.weight": W[f"o_w_{i}"],
                   p + "post_attention_layernorm.weight": norm(W[f"post_attn_ln_w_{i}"]),
                   p + "pre_feedforward_layernorm.weight": norm(W[f"pre_mlp_ln_w_{i}"]),
                   p + "post_feedforward_layernorm.weight": norm(W[f"post_mlp_ln_w_{i}"]),
                   p + "mlp.gate_proj.weight": W[f"gate_w_{i}"], p + "mlp.up_proj.weight": W[f"up_w_{i}"],
                   p + "mlp.down_proj.weight": W[f"down_w_{i}"]})
        if plain:
            sd[p + "self_attn.q_norm.weight"] = norm(W[f"q_norm_w_{i}"])
            sd[p + "self_attn.k_norm.weight"] = norm(W[f"k_norm_w_{i}"])
    return sd


def _gemma_common(cfg):
    return dict(vocab_size=cfg.vocab, hidden_size=cfg.d_model, intermediate_size=cfg.mlp,
                num_hidden_layers=cfg.layers, num_attention_heads=cfg.n_heads,
                num_key_value_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, rms_norm_eps=1e-6,
                sliding_window=cfg.window + 1, attn_implementation="eager", max_position_embeddings=64,
                hidden_activation="gelu_pytorch_tanh")


@pytest.mark.parametrize("B", BATCHES)
def test_gemma2_matches_hf(B):
    from transformers import Gemma2Config, Gemma2ForCausalLM
    # window 4 < prompt 10: local layers (even indices) mask, the global one does not
    cfg = dataclasses.replace(d.GEMMA2_2B, vocab=128, d_model=64, layers=2, n_heads=4, n_kv_heads=2,
                              head_dim=16, mlp=96, window=4, dtype="f32")
    w = d.make_weights(cfg)
    W = dict(zip([n for n, _, _ in d.weight_specs(cfg)], w))
    toks = d.make_prompt(cfg, B, S + DECODE)
    hc = Gemma2Config(attn_logit_softcapping=cfg.attn_softcap, final_logit_softcapping=cfg.final_softcap,
                      query_pre_attn_scalar=cfg.head_dim, **_gemma_common(cfg))
    ref = hf_logits(Gemma2ForCausalLM(hc).eval(), _gemma_state(cfg, W), toks)
    got = oracle_logits(cfg, w, toks)
    assert approx_equal(got, ref), float(np.abs(got - ref).max())


@pytest.mark.parametrize("B", BATCHES)
def test_gemma3_matches_hf(B):
    from transformers import Gemma3ForCausalLM, Gemma3TextConfig
    # 6 layers: five local (window 4, RoPE 1e4) and one global (RoPE 1e6)
    cfg = dataclasses.replace(d.GEMMA3_4B, vocab=128, d_model=64, layers=6, n_heads=4, n_kv_heads=2,
                              head_dim=16, mlp=96, window=4, dtype="f32")
    w = d.make_weights(cfg)
    W = dict(zip([n for n, _, _ in d.weight_specs(cfg)], w))
    toks = d.make_prompt(cfg, B, S + DECODE)
    rope = {"full_attention": {"rope_type": "default", "rope_theta": 1e6},
            "sliding_attention": {"rope_type": "default", "rope_theta": 1e4}}
    hc = Gemma3TextConfig(attn_logit_softcapping=None, final_logit_softcapping=None, query_pre_attn_scalar=1,
                          rope_parameters=rope, **_gemma_common(cfg))
    assert [hc.layer_types[i] == "sliding_attention" for i in range(cfg.layers)] == \
        [cfg.is_local(i) for i in range(cfg.layers)]
    model = Gemma3ForCausalLM(hc).eval()

    class NormedV(torch.nn.Module):
        """V projection followed by gemma.clj:167's weightless RMS norm over kv_dim."""

        def __init__(self, lin):
            super().__init__()
            self.lin = lin

        def forward(self, x):
            v = self.lin(x)
            return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6)

    for layer in model.model.layers:
        layer.self_attn.v_proj = NormedV(layer.self_attn.v_proj)
    ref = hf_logits(model, _gemma_state(cfg, W), toks)
    got = oracle_logits(cfg, w, toks)
    assert approx_equal(got, ref), float(np.abs(got - ref).max())
