"""Tensor-parallel decoding on 2 B200s (one process per GPU, NCCL all-reduce
inside each rank's executable) against the oracle's tensor-parallel executor
running the same shard graphs.  Skipped with fewer than 2 GPUs."""
import dataclasses
import multiprocessing as mp

import numpy as np
import pytest

import conftest  # noqa: F401  - registers the cljxla_b200 package (also in spawned ranks)
from cljxla_b200.host import core, drivers as d, tp
from oracle import interp

from parity import close, close_model, close_model_floor

pytestmark = pytest.mark.gpu

TINY3 = dataclasses.replace(d.GEMMA3_4B, vocab=512, d_model=256, layers=6, n_heads=4, n_kv_heads=2,
                            head_dim=64, mlp=512, window=6)
NOISE_SEEDS = (1, 2, 3, 4)


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank(rank, world, nid, cfg_full, prompt, T, steps, q, hq=None, hin=None):
    try:
        ctx = core.init_tp_backend(world, rank, nid, device=rank)
        if hq is not None:  # one-shot peer all-reduce: handles through the parent
            hq.put((rank, core.p2p_export(ctx)))
            core.p2p_import(ctx, hin.get(timeout=300))
        cfg, gp, gd = tp.shard_graphs(cfg_full, world, prompt.shape[0], prompt.shape[1], T)
        w = d.shard_weights(cfg_full, d.make_weights(cfg_full), rank, world)
        toks, logits = tp.greedy_generate(ctx, cfg, gp, gd, w, prompt, T, steps)
        core.close_backend(ctx)
        q.put((rank, toks, logits, None))
    except Exception as e:  # noqa: BLE001 - reported by the parent
        q.put((rank, None, None, repr(e)))


def _run_group(cfg_full, world, prompt, T, steps, p2p=False):
    nid = core.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    hq = ctx.Queue() if p2p else None
    hins = [ctx.Queue() for _ in range(world)] if p2p else [None] * world
    procs = [ctx.Process(target=_rank, args=(r, world, nid, cfg_full, prompt, T, steps, q, hq, hins[r]))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        if p2p:
            hs = dict(hq.get(timeout=300) for _ in range(world))
            for hin in hins:
                hin.put([hs[r] for r in range(world)])
        for _ in range(world):
            r, toks, logits, err = q.get(timeout=600)
            assert err is None, f"rank {r}: {err}"
            res[r] = (toks, logits)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    return res


@pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("dtype,p2p", [("f32", False), ("bf16", False), ("f32", True), ("bf16", True)])
def test_tp2_greedy_decode_matches_oracle(dtype, p2p):
    """2-rank decode against the sharded oracle, the all_reduce ops on NCCL or
    (p2p) on the one-shot kernel over NVLink peer memory (rank-order sum)."""
    cfg = dataclasses.replace(TINY3, dtype=dtype)
    B, S, T, steps = 1, 6, 32, 12
    prompt = d.make_prompt(cfg, B, S)
    w = d.make_weights(cfg)
    res = _run_group(cfg, 2, prompt, T, steps, p2p)
    o_toks, o_logits = tp.oracle_generate(cfg, 2, w, prompt, T, steps, interp.run_mlir_tp, interp.run_mlir)
    # every rank holds the same all-reduced logits and picks the same tokens
    assert res[0][0] == res[1][0]
    for a, b in zip(res[0][1], res[1][1]):
        assert np.array_equal(a, b)
    assert res[0][0] == o_toks
    floors = None
    for i, (a, b) in enumerate(zip(res[0][1], o_logits)):
        if dtype == "f32":
            ok, excess, err = close(a, b, "f32")
            assert ok, f"step {i}: f32 logits differ, max err {err:.3g}"
            continue
        else:
            ok, bad, rr = close_model(a, b, "bf16")
            if not ok:
                if floors is None:
                    floors = [tp.oracle_generate(
                        cfg, 2, w, prompt, T, steps,
                        lambda texts, ins, sd=sd: interp.run_mlir_tp(texts, ins, ulp_noise_seed=sd),
                        interp.run_mlir)[1] for sd in NOISE_SEEDS]
                ok, bad, rr, fb, fr = close_model_floor(a, b, [f[i] for f in floors], "bf16")
        assert ok, f"step {i}: {bad:.2%} out of bound, rel rms {rr:.3g} (floor {fb:.2%}, {fr:.3g})"


def _rank_vocab(rank, world, nid, cfg_full, shape, ins, q):
    try:
        from cljxla_b200.host import runner
        ctx = core.init_tp_backend(world, rank, nid, device=rank)
        B, S, T = shape
        g = d.build_graph(d.shard_config(cfg_full, world, vocab_rank=rank), "decode", B, S, T, greedy=True)
        out = runner.run_graph(ctx, g, ins)
        core.close_backend(ctx)
        q.put((rank, np.asarray(out[0]), None))
    except Exception as e:  # noqa: BLE001 - reported by the parent
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("tie", [False, True], ids=["random", "all-tied"])
def test_tp2_vocab_split_greedy_token(tie):
    """A greedy decode step whose LM head is split by vocabulary rows over 2
    ranks: the token the two max all-reduces (NCCL, f32 values and i32
    indices) agree on equals the sharded oracle's, on both ranks, and the
    all-tied step gives the last index."""
    from test_tp import _split_decode_inputs
    cfg = dataclasses.replace(TINY3, dtype="f32")
    B, S, T, world = 2, 6, 16, 2
    ins = _split_decode_inputs(cfg, B, S, T, world, tie=tie)
    from cljxla_b200.host import stablehlo as shlo
    texts = [shlo.graph_to_mlir_text(d.build_graph(d.shard_config(cfg, world, vocab_rank=r), "decode", B, S, T,
                                                   greedy=True)) for r in range(world)]
    want = np.asarray(interp.run_mlir_tp(texts, ins)[0][0])
    nid = core.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_vocab, args=(r, world, nid, cfg, (B, S, T), ins[r], q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, tok, err = q.get(timeout=300)
            assert err is None, f"rank {r}: {err}"
            got[r] = tok
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert np.array_equal(got[r], want), (r, got[r].ravel(), want.ravel())
    if tie:
        assert np.all(want == cfg.vocab - 1)


def _rank_skip(rank, world, nid, q, hq, hin, go, ready, start):
    """Rank of a 2-rank group whose rank 1 leaves after the first step."""
    import os
    os.environ["CLJXLA_B200_P2P_WAIT_POLLS"] = "500000"  # about half a second before a wait gives up
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from cljxla_b200.host import stablehlo as shlo
    from cljxla_b200.host import tensor as t
    from cljxla_b200.host.pjrt import PJRTError
    try:
        ctx = core.init_tp_backend(world, rank, nid, device=rank)
        hq.put((rank, core.p2p_export(ctx)))
        core.p2p_import(ctx, hin.get(timeout=300))
        g = t.trace_graph("ar", [("x", ("tensor", (1, 64), "f32"))], lambda x: [t.all_reduce(x, 2)])
        exe = core.compile_mlir_text(ctx, shlo.graph_to_mlir_text(g), g)
        x = np.full((1, 64), rank + 1.0, np.float32)

        def step():
            b = core.buffer_from_host_buffer(ctx, x, (1, 64), 11)
            try:
                out = ctx["api"].execute_executable(exe["handle"], [b], 1)
                try:
                    return core.buffer_to_numpy(ctx, out, (1, 64), "f32")
                finally:
                    core.destroy_buffer(ctx, out)
            finally:
                core.destroy_buffer(ctx, b)

        ready.put(rank)  # both ranks start the first step together (compile times differ)
        start.get(timeout=300)
        first = step()
        ok = bool(np.all(first == 3.0))
        if rank == 1:  # leaves between steps, nothing in flight, and waits for the end
            q.put((rank, ok, "left"))
            go.get(timeout=300)
            core.close_backend(ctx)
            return
        step()  # the peer never arrives: the kernel's bounded wait runs out and it returns
        try:
            step()
            msg = "no error"
        except PJRTError as e:
            msg = str(e)
        core.close_backend(ctx)
        q.put((rank, ok, msg))
    except Exception as e:  # noqa: BLE001 - reported by the parent
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")
def test_p2p_wait_runs_out_when_a_rank_leaves():
    """A rank leaves the group between steps; the other rank's one-shot
    all-reduce waits a short, bounded time for its flag, gives up, and the
    next execution on that rank reports the group out of step as a PJRT
    error - the GPU and the context stay usable (the client closes cleanly)."""
    nid = core.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q, hq, go, ready = ctx.Queue(), ctx.Queue(), ctx.Queue(), ctx.Queue()
    hins = [ctx.Queue() for _ in range(2)]
    starts = [ctx.Queue() for _ in range(2)]
    procs = [ctx.Process(target=_rank_skip, args=(r, 2, nid, q, hq, hins[r], go, ready, starts[r]))
             for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        hs = dict(hq.get(timeout=300) for _ in range(2))
        for hin in hins:
            hin.put([hs[r] for r in range(2)])
        for _ in range(2):
            ready.get(timeout=300)
        for st in starts:
            st.put("go")
        for _ in range(2):
            r, ok, msg = q.get(timeout=300)
            res[r] = (ok, msg)
            if r == 0:
                go.put("done")
    finally:
        go.put("done")
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert res[0][0] and res[1][0], res
    assert res[1][1] == "left"
    assert "out of step" in res[0][1], res[0][1]
