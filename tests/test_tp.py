"""Tensor parallelism, host side (no device): shard configs and weights, the
printed all_reduce, planning of shard graphs by the library, the oracle's
tensor-parallel executor against the unsharded model, and sharing of the NCCL
id over a 2-rank gloo group."""
import dataclasses
import multiprocessing as mp
import os
import re
import socket

import numpy as np
import pytest

import conftest  # noqa: F401  - registers the cljxla_b200 package (also in spawned ranks)
from cljxla_b200.host import core, drivers as d, tp
from cljxla_b200.host import stablehlo as shlo
from oracle import interp

from parity import close

TINY3 = dataclasses.replace(d.GEMMA3_4B, vocab=512, d_model=256, layers=6, n_heads=4, n_kv_heads=2,
                            head_dim=64, mlp=512, window=6)
TINY2 = dataclasses.replace(d.GEMMA2_2B, vocab=512, d_model=256, layers=2, n_heads=4, n_kv_heads=2,
                            head_dim=64, mlp=512, window=6)


@pytest.fixture(scope="module")
def lib_path():
    import __graft_entry__
    __graft_entry__.build()
    from cljxla_b200 import LIB_PATH
    return LIB_PATH


def test_shard_config_divides_heads_and_mlp():
    c = d.shard_config(d.GEMMA3_27B, 8)
    assert (c.n_heads, c.n_kv_heads, c.mlp, c.tp) == (4, 2, 21504 // 8, 8)
    assert c.d_model == d.GEMMA3_27B.d_model and c.vocab == d.GEMMA3_27B.vocab
    with pytest.raises(ValueError):
        d.shard_config(d.GEMMA3_4B, 8)          # 4 KV heads do not split 8 ways
    with pytest.raises(ValueError):
        d.shard_config(d.GPT2_SMALL, 2)


def test_row_and_column_split_reassemble_the_projection():
    """Column split of q/gate (output rows) and row split of o/down (input
    columns): the ranks' partial products sum to the unsharded product."""
    full = d.make_weights(TINY3)
    specs = d.weight_specs(TINY3)
    ws = [d.shard_weights(TINY3, full, r, 2) for r in range(2)]
    idx = {n: i for i, (n, _, _) in enumerate(specs)}
    q, o = idx["q_w_0"], idx["o_w_0"]
    f32 = interp.bf16_bits_to_f32
    assert np.array_equal(np.concatenate([f32(ws[0][q]), f32(ws[1][q])], 0), f32(full[q]))
    x = np.random.default_rng(0).standard_normal((3, full[o].shape[1])).astype(np.float32)
    half = full[o].shape[1] // 2
    parts = sum(x[:, r * half:(r + 1) * half] @ f32(ws[r][o]).T for r in range(2))
    np.testing.assert_allclose(parts, x @ f32(full[o]).T, rtol=1e-5, atol=1e-5)
    # replicated weights are the same objects' values
    e = idx["embed_tokens"]
    assert np.array_equal(ws[1][e], full[e])


@pytest.mark.parametrize("cfg", [TINY3, TINY2], ids=["gemma3", "gemma2"])
def test_printed_shard_graph_has_all_reduces(cfg):
    sc = d.shard_config(cfg, 2)
    txt = shlo.graph_to_mlir_text(d.build_graph(sc, "decode", 1, 8, 16))
    n = len(re.findall(r'"stablehlo\.all_reduce"\(', txt))
    # o-projection and down-projection per layer; Gemma-3 adds the V-norm sum of squares
    per_layer = 3 if cfg.family == "gemma3" else 2
    assert n == per_layer * cfg.layers
    assert "replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>" in txt
    assert "stablehlo.add" in txt.split('"stablehlo.all_reduce"(', 1)[1].split("})", 1)[0]


def test_library_plans_shard_graphs(lib_path):
    sc = d.shard_config(d.GEMMA3_27B, 8)
    for kind in ("decode", "prefill"):
        g = d.build_graph(sc, kind, 1, 16, 128, dynamic_prefill=kind == "prefill")
        info = core.plan_text(lib_path, shlo.graph_to_mlir_text(g), 3)
        assert info["launches"] >= 3 * sc.layers


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_tp_oracle_matches_unsharded_oracle(dtype):
    """The 2-rank oracle (f64 rank-order sums) decodes the same greedy tokens
    as the unsharded graph.  In f32 the logits agree to the f32 tolerance (the
    sharding only reorders sums); in bf16 each rank rounds its partial
    projection to bf16 before the sum, a different rounding than one bf16
    rounding of the whole dot, so only a loose bound holds there."""
    cfg = dataclasses.replace(TINY3, dtype=dtype)
    w = d.make_weights(cfg)
    prompt = d.make_prompt(cfg, 1, 6)
    t1, l1 = tp.oracle_generate(cfg, 1, w, prompt, 16, 5, interp.run_mlir_tp, interp.run_mlir)
    t2, l2 = tp.oracle_generate(cfg, 2, w, prompt, 16, 5, interp.run_mlir_tp, interp.run_mlir)
    assert t1 == t2
    for a, b in zip(l2, l1):
        if dtype == "f32":
            ok, excess, err = close(a, b, "f32")
            assert ok, (excess, err)
        else:
            rr = float(np.sqrt(np.mean((a - b) ** 2)) / np.sqrt(np.mean(b ** 2)))
            assert rr < 0.05, rr


def _split_decode_inputs(cfg, B, S, T, tp_n, seed=3, tie=False):
    w = d.make_weights(cfg)
    if tie:   # final (1 + w) norm weight -1: every logit is 0, the argmax is the last index
        i = [n for n, _, _ in d.weight_specs(cfg)].index("final_norm_w")
        w[i] = np.full_like(w[i], 0xBF80 if cfg.dtype == "bf16" else -1.0)
    rng = np.random.default_rng(seed)
    kv = [rng.standard_normal(d.cache_shape(cfg, B, T)).astype(np.float32) for _ in range(2 * cfg.layers)]
    if cfg.dtype == "bf16":
        kv = [d._to_bf16_bits(a) for a in kv]
    toks = d.make_prompt(cfg, B, 1, seed=seed)
    pos = d.pos_inputs(cfg, "decode", B, S, 1)
    nk = cfg.n_kv_heads // tp_n
    return [[toks, pos] + d.shard_weights(cfg, w, r, tp_n) + [a[:, r * nk:(r + 1) * nk].copy() for a in kv]
            for r in range(tp_n)]


@pytest.mark.parametrize("cfg,tie", [(dataclasses.replace(TINY3, dtype="f32"), False), (TINY3, False),
                                     (TINY2, False), (TINY3, True)],
                         ids=["gemma3-f32", "gemma3-bf16", "gemma2-softcap", "all-tied"])
def test_vocab_split_greedy_matches_replicated_head(cfg, tie, lib_path):
    """Greedy decode graphs with the LM head split by vocabulary rows pick the
    same token on every rank as the replicated head, which every rank
    computes in full: each logit is the same dot either way, and the two max
    all-reduces keep the in-graph argmax's highest-index tie rule (the
    all-tied case must give V - 1).  The library plans the split graphs."""
    B, S, T, n = 2, 6, 16, 2
    ins = _split_decode_inputs(cfg, B, S, T, n, tie=tie)
    rep = shlo.graph_to_mlir_text(d.build_graph(d.shard_config(cfg, n), "decode", B, S, T, greedy=True))
    want = interp.run_mlir_tp([rep] * n, ins)
    texts = [shlo.graph_to_mlir_text(d.build_graph(d.shard_config(cfg, n, vocab_rank=r), "decode", B, S, T,
                                                   greedy=True)) for r in range(n)]
    assert texts[0] != texts[1]                       # the ranks slice different vocabulary rows
    assert len(re.findall(r"%arg_res = stablehlo.maximum %arg_a, %arg_b : tensor<(f32|i32)>", texts[0])) >= 2
    got = interp.run_mlir_tp(texts, ins)
    for r in range(n):
        assert np.array_equal(got[r][0], want[0][0]), (r, got[r][0].ravel(), want[0][0].ravel())
    if tie:
        assert np.all(np.asarray(got[0][0]) == cfg.vocab - 1)
    for r in range(n):
        assert core.plan_text(lib_path, texts[r])["launches"] > 0


def test_vocab_split_head_reads_its_rows_only(lib_path, tmp_path):
    """The planned LM-head launch of a vocab-split rank reads V / tp rows of
    the tied embedding in place: its algorithmic bytes are half the
    replicated head's at tp = 2 (the embedding dominates both), with no copy
    of the slice."""
    cfg = dataclasses.replace(TINY3, vocab=8192)
    biggest = {}
    for name, vr in (("replicated", None), ("split", 1)):
        dump = tmp_path / f"{name}.txt"
        txt = shlo.graph_to_mlir_text(d.build_graph(d.shard_config(cfg, 2, vocab_rank=vr), "decode", 1, 6, 16,
                                                    greedy=True))
        code = ("import sys; sys.path.insert(0, %r); import __graft_entry__ as g; g._pkg();"
                "from cljxla_b200.host import core; core.plan_text(%r, sys.stdin.read())"
                % (os.path.dirname(os.path.dirname(os.path.abspath(__file__))), lib_path))
        import subprocess
        import sys
        r = subprocess.run([sys.executable, "-c", code], input=txt, capture_output=True, text=True, timeout=300,
                           env=dict(os.environ, CLJXLA_B200_DUMP_PLAN=str(dump)))
        assert r.returncode == 0, r.stderr[-2000:]
        rows = [ln.split("\t") for ln in dump.read_text().splitlines() if not ln.startswith("#")]
        assert not any(k == "copy" and int(b) >= cfg.vocab * cfg.d_model for k, b, _ in rows)
        biggest[name] = max(int(b) for _, b, _ in rows)
    table = cfg.vocab * cfg.d_model * 2
    assert biggest["replicated"] >= table
    assert table // 2 <= biggest["split"] < table // 2 + table // 16


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gloo_rank(rank, world, port, lib, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, tp.share_nccl_id(lib)))
    finally:
        dist.destroy_process_group()


def test_nccl_id_shared_over_two_gloo_ranks(lib_path):
    try:
        core.nccl_unique_id(lib_path)
    except RuntimeError:
        pytest.skip("NCCL not loadable on this host")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, lib_path, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=90) for _ in range(2))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert set(got) == {0, 1}
    assert got[0] == got[1] and len(got[0]) == 256 and int(got[0], 16) >= 0


def _gloo_rank_failing_nccl(rank, world, port, lib, q):
    import datetime
    import torch.distributed as dist
    if rank == 0:  # the injected failure: rank 0's NCCL cannot be loaded
        os.environ["CLJXLA_B200_NCCL_LIB"] = "/nonexistent/libnccl.so.2"
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        tp.share_nccl_id(lib)
        q.put((rank, "joined"))
    except tp.GroupError as e:
        q.put((rank, "GroupError: " + str(e)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_nccl_init_failure_reaches_every_gloo_rank(lib_path):
    """An NCCL that cannot be loaded on rank 0 (injected through
    CLJXLA_B200_NCCL_LIB) ends the group set-up on both ranks with GroupError,
    naming the cause, well before the process group's timeout."""
    import time
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank_failing_nccl, args=(r, 2, port, lib_path, q)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=90) for _ in range(2))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert set(got) == {0, 1}
    for r in (0, 1):
        assert got[r].startswith("GroupError") and "NCCL" in got[r], got
    assert time.time() - t0 < 60
