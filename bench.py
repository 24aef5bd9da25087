"""Decode / prefill throughput of the clj-xla decoder path on B200.

Workload (default): Gemma-3-4B bf16, random-init weights, batch 1, prompt 2048
random token ids, KV cache of 2048+512 positions - the headline HBM-roofline
configuration.  A *step* is one KV-cached decode step of the whole model
(one token per sequence): the lowered StableHLO decode graph executed by
libcljxla_b200.so through its PJRT C ABI.  ``value`` is decode tokens/s with
each step's token / position buffers already on the device; ``e2e`` is the
same loop driven the way clj-xla's host drives it (upload token and position
from host memory, execute, read the f32 logits back, greedy argmax on the
host).  Prefill tokens/s of the same model is reported in ``prefill``.

With ``--gpus N`` (torchrun, one process per GPU) every rank runs an
independent replica of the workload (data parallel, no collective on the data
path; ``scaling: weak``); value = all ranks' tokens / max time over ranks.
With ``--tp N`` (torchrun with N ranks) the ranks instead hold the N shards of
one model (Gemma: heads and MLP split, an NCCL all-reduce after the attention
and MLP blocks; ``scaling: strong``), e.g. ``--config gemma3-12b --tp 4``.

``--impl reference`` times the CPU restatement of the reference's execution
path (oracle/interp.py running the same printed graph on the host cores).
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))


def _pkg():
    import importlib.util
    if "cljxla_b200" in sys.modules:
        return sys.modules["cljxla_b200"]
    pkg_dir = os.path.join(ROOT, "clj-xla_b200")
    spec = importlib.util.spec_from_file_location(
        "cljxla_b200", os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["cljxla_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=32)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default="gemma3-4b")
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--prompt", type=int, default=2048)
    p.add_argument("--gen", type=int, default=512)
    p.add_argument("--prefill-reps", type=int, default=3)
    p.add_argument("--e2e-steps", type=int, default=16)
    p.add_argument("--cpu-steps", type=int, default=1)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--tiny", action="store_true", help="reduced model for quick checks (not a bench line)")
    p.add_argument("--decode-only", action="store_true",
                   help="only the decode steps (zero caches, no prefill / e2e / profile): for ncu launch lists")
    p.add_argument("--profile", action="store_true",
                   help="with --decode-only: also print per-kind device time of a profiled step")
    p.add_argument("--layers", type=int, default=0,
                   help="override the layer count (small ncu captures; not a bench line)")
    p.add_argument("--tp", type=int, default=1,
                   help="tensor-parallel ranks per model replica (Gemma; ranks = --gpus under torchrun)")
    p.add_argument("--no-tp-block", action="store_true",
                   help="skip the tensor-parallel Gemma-3-12B batch-8 decode measurement added to the line")
    p.add_argument("--tp-steps", type=int, default=16)
    return p.parse_args()


def tp_block(args, rank, world, local_rank):
    """Gemma-3-12B bf16 batch 8 decode (prompt 4096, KV cache 4608 positions),
    tensor-parallel over every rank of the job (TP = world; one GPU: TP 1).
    Each rank holds its shard (heads and MLP width split, an all-reduce after
    the attention and MLP blocks: the one-shot peer kernel for messages that
    fit its slot, NCCL above), weights random-init on the device, caches
    zero, the decode graph replayed at positions 4096 + i with device-resident
    token ids.  Returns the device time per step (max over ranks)."""
    import torch
    from cljxla_b200.host import core, drivers as d
    from cljxla_b200.host import stablehlo as shlo
    from cljxla_b200.host.pjrt import DTYPE_ENUM
    pkg = _pkg()
    cfg_full, B, S = d.GEMMA3_12B, 8, 4096
    T = d.round_up(S + 512, 128)
    cfg = d.shard_config(cfg_full, world)
    if world > 1:
        from cljxla_b200.host import tp as tpmod
        ctx = core.init_tp_backend(world, rank, tpmod.share_nccl_id(pkg.LIB_PATH), local_rank, pkg.LIB_PATH)
        tpmod.setup_p2p(ctx, 128 << 10)  # a [8, 3840] bf16 block sum (61 KB) fits one slot
    else:
        ctx = core.init_backend(pkg.LIB_PATH, {"device": local_rank})
    api = ctx["api"]
    wdt = DTYPE_ENUM[cfg.dtype]
    host_w = d.device_weights(cfg, 4321 + rank, f"cuda:{local_rank}")
    wbufs = [core.buffer_from_host_buffer(ctx, w, shp, wdt) for w, (_, shp, _) in zip(host_w, d.weight_specs(cfg))]
    del host_w
    g = d.build_graph(cfg, "decode", B, S, T)
    ex = core.compile_mlir_text(ctx, shlo.graph_to_mlir_text(g), g)
    cache = d.zero_cache(cfg, B, T)
    kv = [core.buffer_from_host_buffer(ctx, cache, list(cache.shape), wdt) for _ in range(2 * cfg.layers)]
    n = args.warmup + args.tp_steps
    rng = np.random.Generator(np.random.PCG64(11))  # the same ids on every rank
    xs = [core.buffer_from_host_buffer(ctx, rng.integers(0, cfg.vocab, size=(B, 1), dtype=np.int64).astype(np.int32),
                                       [B, 1], 4) for _ in range(n)]
    ps = [core.buffer_from_host_buffer(ctx, np.array([S + i], np.int32), [1], 4) for i in range(n)]
    stream = torch.cuda.ExternalStream(core.client_stream(ctx), device=f"cuda:{local_rank}")

    def step(i, kv):
        outs = api.execute_executable(ex["handle"], [xs[i], ps[i]] + wbufs + kv, len(g["outvars"]), wait=False)
        api.destroy_buffer(outs[0])
        for b in kv:
            api.destroy_buffer(b)
        return outs[1:]

    for i in range(args.warmup):
        kv = step(i, kv)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.warmup, n):
        kv = step(i, kv)
    e1.record(stream)
    e1.synchronize()
    dt = e0.elapsed_time(e1) / 1e3
    if world > 1:
        t = torch.tensor([dt], device=f"cuda:{local_rank}")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dt = float(t.item())
    plan = core.plan_info(ctx, ex)
    for b in kv + xs + ps + wbufs:
        api.destroy_buffer(b)
    core.close_backend(ctx)
    ms = dt / args.tp_steps * 1e3
    # per-GPU weight bytes streamed per step (the decode is HBM-bound): the
    # shard's weights once per step, over the measured copy bandwidth
    w_bytes = sum(int(np.prod(shp)) for _, shp, _ in d.weight_specs(cfg)) * 2
    hbm, _, src = load_peaks()
    return {"config": "gemma3-12b decode, batch 8, prompt 4096, KV cache 4608 positions", "tp": world,
            "ms_per_step": round(ms, 4), "tokens_per_s": round(B * args.tp_steps / dt, 2),
            "weight_bytes_per_gpu": w_bytes, "weight_floor_ms": round(w_bytes / (hbm * 1e9) * 1e3, 4),
            "steps": args.tp_steps, "launches_per_step": plan["launches"],
            "timing": "CUDA events on each rank's stream, max over ranks"}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), float(pk["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    def __init__(self, gpu_index, period_ms=20):
        self.gpu = gpu_index
        self.period = period_ms
        self.proc = None
        self.lines = []  # (host time, csv line)
        self.window = None

    def wait_first(self, timeout=3.0):
        """nvidia-smi needs a moment before its first line: start the sampler
        early and wait for it, so samples cover the timed region."""
        t_end = time.perf_counter() + timeout
        while self.proc and not self.lines and time.perf_counter() < t_end:
            time.sleep(0.01)

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.period)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append((time.perf_counter(), ln.strip()))

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = [ln for t, ln in self.lines
                 if self.window is None or self.window[0] - 0.03 <= t <= self.window[1] + 0.03]
        for ln in lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "period_ms": self.period}


def model_setup(args):
    from cljxla_b200.host import drivers as d
    import dataclasses
    cfg = d.CONFIGS[args.config]
    if args.tiny:
        cfg = dataclasses.replace(cfg, vocab=2048, d_model=256, layers=4, n_heads=4, n_kv_heads=2, head_dim=64,
                                  mlp=1024, window=64)
    if args.layers:
        cfg = dataclasses.replace(cfg, layers=args.layers)
    B, S = args.batch, args.prompt
    T = d.round_up(S + args.gen, 128)
    return cfg, B, S, T


def run_ours(args, rank, world, local_rank):
    import torch
    pkg = _pkg()
    from cljxla_b200.host import core, drivers as d
    from cljxla_b200.host import stablehlo as shlo
    from cljxla_b200.host.pjrt import DTYPE_ENUM

    torch.cuda.set_device(local_rank)
    cfg_full, B, S, T = model_setup(args)
    cfg = d.shard_config(cfg_full, args.tp)
    if args.tp > 1:
        from cljxla_b200.host import tp as tpmod
        ctx = core.init_tp_backend(args.tp, rank % args.tp, tpmod.share_nccl_id(pkg.LIB_PATH), local_rank,
                                   pkg.LIB_PATH)
        if os.environ.get("CLJXLA_B200_P2P", "1") != "0":
            tpmod.setup_p2p(ctx)  # small all_reduce ops: one-shot kernel over NVLink peer memory
    else:
        ctx = core.init_backend(pkg.LIB_PATH, {"device": local_rank})
    api, client = ctx["api"], ctx["client"]
    wdt = DTYPE_ENUM[cfg.dtype]

    t0 = time.time()
    host_w = d.device_weights(cfg, 1234 + rank, f"cuda:{local_rank}")
    specs = d.weight_specs(cfg)
    wbufs = [core.buffer_from_host_buffer(ctx, w, shp, wdt) for w, (_, shp, _) in zip(host_w, specs)]
    if args.no_cpu_baseline or rank != 0 or args.tp > 1:
        del host_w
        host_w = None
    t_w = time.time() - t0

    g_dec = d.build_graph(cfg, "decode", B, S, T)
    g_pre = d.build_graph(cfg, "prefill", B, S, T, dynamic_prefill=True)
    txt_dec, txt_pre = shlo.graph_to_mlir_text(g_dec), shlo.graph_to_mlir_text(g_pre)
    t1 = time.time()
    ex_dec = core.compile_mlir_text(ctx, txt_dec, g_dec)
    # (decode-only runs never execute the prefill graph, whose scratch can be large)
    ex_pre = None if args.decode_only else core.compile_mlir_text(ctx, txt_pre, g_pre)
    # the same decode step with in-graph greedy sampling (tensor.clj:519-532):
    # what a user's generation loop runs, reading 4 bytes per sequence per step
    g_greedy = d.build_graph(cfg, "decode", B, S, T, greedy=True) if cfg.family != "gpt2" else None
    ex_greedy = core.compile_mlir_text(ctx, shlo.graph_to_mlir_text(g_greedy), g_greedy) if g_greedy else None
    t_c = time.time() - t1

    cache_np = d.zero_cache(cfg, B, T)
    cshape = list(cache_np.shape)

    def zero_kv():
        return [core.buffer_from_host_buffer(ctx, cache_np, cshape, wdt) for _ in range(2 * cfg.layers)]

    stream = torch.cuda.ExternalStream(core.client_stream(ctx), device=f"cuda:{local_rank}")
    rng = np.random.Generator(np.random.PCG64(7 + rank))

    # ---------------- prefill (dynamic-position prefill graph, one sequence batch)
    toks = d.make_prompt(cfg, B, S, seed=1 + rank)
    x_pre = core.buffer_from_host_buffer(ctx, toks, [B, S], 4)
    pos_pre = d.pos_inputs(cfg, "prefill", B, 0, S)
    p_pre = core.buffer_from_host_buffer(ctx, pos_pre, list(pos_pre.shape), 4)
    pre_times = []
    kv = None
    if args.decode_only:
        kv = zero_kv()
        pre_times = [float("nan")]
    for rep in range(0 if args.decode_only else max(1, args.prefill_reps) + 1):
        kv0 = zero_kv()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        outs = api.execute_executable(ex_pre["handle"], [x_pre, p_pre] + wbufs + kv0, len(g_pre["outvars"]), wait=False)
        e1.record(stream)
        e1.synchronize()
        if rep > 0:
            pre_times.append(e0.elapsed_time(e1) / 1e3)
        for b in kv0:
            api.destroy_buffer(b)
        api.destroy_buffer(outs[0])
        if kv is not None:
            for b in kv:
                api.destroy_buffer(b)
        kv = outs[1:]
    prefill_s = float(np.median(pre_times))
    # one profiled prefill (per-kernel events): where the prefill time goes
    pre_by_kind = {}
    if not args.decode_only:
        kvp = zero_kv()
        core.profile_enable(ctx, True)
        outs = api.execute_executable(ex_pre["handle"], [x_pre, p_pre] + wbufs + kvp, len(g_pre["outvars"]))
        torch.cuda.synchronize()
        for e in core.profile_dump(ctx):
            pre_by_kind[e["kind"]] = round(pre_by_kind.get(e["kind"], 0.0) + e["ms"], 3)
        core.profile_enable(ctx, False)
        for b in kvp + outs:
            api.destroy_buffer(b)

    # ---------------- decode, device-resident inputs
    n_total = args.warmup + args.steps
    xs = [core.buffer_from_host_buffer(ctx, rng.integers(0, cfg.vocab, size=(B, 1), dtype=np.int64).astype(np.int32),
                                       [B, 1], 4) for _ in range(n_total)]
    def pos_buf(pos):  # the decode step's position invar ([1], or [B, 1] for GPT-2)
        a = d.pos_inputs(cfg, "decode", B, pos, 1)
        return core.buffer_from_host_buffer(ctx, a, list(a.shape), 4)

    ps = [pos_buf(S + (i % (T - S))) for i in range(n_total)]

    def step(i, kv):
        outs = api.execute_executable(ex_dec["handle"], [xs[i], ps[i]] + wbufs + kv, len(g_dec["outvars"]), wait=False)
        api.destroy_buffer(outs[0])
        for b in kv:
            api.destroy_buffer(b)
        return outs[1:]

    with ClockSampler(local_rank) as clk:
        clk.wait_first()
        for i in range(args.warmup):
            kv = step(i, kv)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        launches0 = core.kernel_launches(ctx)
        h0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.warmup, n_total):
            kv = step(i, kv)
        e1.record(stream)
        e1.synchronize()
        clk.mark(h0, time.perf_counter())
        time.sleep(0.05)  # the sample taken at the end of the region
    dec_s = e0.elapsed_time(e1) / 1e3
    launches = core.kernel_launches(ctx) - launches0
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    if args.decode_only:
        line = {"decode_only": True, "ms_per_step": dec_s / args.steps * 1e3, "launches": launches}
        if args.profile:  # per-kind device time of two steps with events around every launch
            core.profile_enable(ctx, True)
            for i in range(2):
                kv = step(i % n_total, kv)
            torch.cuda.synchronize()
            agg = {}
            for e in core.profile_dump(ctx):
                a = agg.setdefault(e["kind"], [0.0, 0, 0])
                a[0] += e["ms"] / 2
                a[1] += e["bytes"] // 2
                a[2] += e["calls"] // 2
            core.profile_enable(ctx, False)
            line["kernel_ms_per_step"] = {k: round(v[0], 4) for k, v in agg.items()}
            line["gb_per_s"] = {k: round(v[1] / (v[0] / 1e3) / 1e9, 1) for k, v in agg.items() if v[0] > 0}
            line["launches_per_step"] = {k: v[2] for k, v in agg.items()}
        print(json.dumps(line))
        for b in kv + xs + ps + wbufs + [x_pre, p_pre]:
            api.destroy_buffer(b)
        return cfg, B, S, T, None

    # ---------------- decode end to end through the PJRT C ABI, the way the
    # host drives it: token and position uploaded from host memory, execute,
    # the step's result read back (which waits for the step), and the previous
    # step's buffers destroyed while this step runs on the device.
    # Headline: the greedy graph (token ids read back, 4 bytes per sequence);
    # also the logits graph with the host argmax of scripts/gemma4_inference.clj.
    logits_bytes = B * cfg.vocab * 4
    e2e_steps = max(1, args.e2e_steps)

    def e2e_loop(greedy, kv):
        tok = np.array([[int(toks[0, -1])]] * B, np.int32)
        ex, g = (ex_greedy, g_greedy) if greedy else (ex_dec, g_dec)
        prev = []
        t_e0 = None
        for i in range(e2e_steps + 2):  # two untimed warm-up steps (the first execution records its CUDA graph)
            if i == 2:
                torch.cuda.synchronize()
                t_e0 = time.perf_counter()
            xb = core.buffer_from_host_buffer(ctx, tok, [B, 1], 4)
            pb = pos_buf(S + (i % (T - S)))
            outs = api.execute_executable(ex["handle"], [xb, pb] + wbufs + kv, len(g["outvars"]), wait=False)
            for b in prev:  # the previous step has completed (its result was read back)
                api.destroy_buffer(b)
            prev = [xb, pb, outs[0]] + kv
            kv = outs[1:]
            if greedy:
                tok = api.buffer_to_host(outs[0], 4 * B).view(np.int32).reshape(B, 1).copy()
            else:
                logits = api.buffer_to_host_floats(outs[0], B * cfg.vocab).reshape(B, cfg.vocab)
                tok = np.array([[d.argmax_host(logits[b])] for b in range(B)], np.int32)
        for b in prev:
            api.destroy_buffer(b)
        torch.cuda.synchronize()
        return time.perf_counter() - t_e0, kv

    e2e_logits_s, kv = e2e_loop(False, kv)
    e2e_s, kv = e2e_loop(True, kv) if ex_greedy else (e2e_logits_s, kv)

    # ---------------- roofline of the dominant kernel (one profiled decode step)
    core.profile_enable(ctx, True)
    for i in range(2):
        kv = step(i % n_total, kv)
    torch.cuda.synchronize()
    prof = core.profile_dump(ctx)
    core.profile_enable(ctx, False)
    by_kind = {}
    for e in prof:
        k = by_kind.setdefault(e["kind"], {"ms": 0.0, "bytes": 0, "flops": 0, "calls": 0})
        k["ms"] += e["ms"]
        k["bytes"] += e["bytes"]
        k["flops"] += e["flops"]
        k["calls"] += e["calls"]
    total_ms = sum(k["ms"] for k in by_kind.values())
    dom = max(by_kind.items(), key=lambda kv_: kv_[1]["ms"])
    hbm_peak, tc_peak, peak_src = load_peaks()
    achieved = dom[1]["bytes"] / (dom[1]["ms"] / 1e3) / 1e9 if dom[1]["ms"] else 0.0

    # ---------------- CPU baseline (rank 0, N=1): oracle on the host cores, bounded sample
    cpu = None
    if rank == 0 and world == 1 and host_w is not None:
        cpu = cpu_baseline(cfg, B, S, T, txt_dec, host_w, args.cpu_steps)

    for b in kv + xs + ps + wbufs + [x_pre, p_pre]:
        api.destroy_buffer(b)
    plan = core.plan_info(ctx, ex_dec)
    core.close_backend(ctx)

    tokens = B * args.steps
    res = {
        "rank": rank, "dec_s": dec_s, "tokens": tokens, "prefill_s": prefill_s, "e2e_s": e2e_s,
        "pre_by_kind": pre_by_kind,
        "e2e_tokens": B * e2e_steps, "launches": launches, "clocks": clk.summary(),
        "by_kind": by_kind, "total_ms": total_ms, "dom": dom[0], "achieved": achieved,
        "hbm_peak": hbm_peak, "peak_src": peak_src, "cpu": cpu, "t_weights": t_w, "t_compile": t_c,
        "plan": plan, "logits_bytes": logits_bytes, "e2e_logits_s": e2e_logits_s,
        "e2e_greedy": ex_greedy is not None,
    }
    return cfg, B, S, T, res


def safe(fn, *a):
    """A derived figure of the line, or its error (the measured values stand)."""
    try:
        return fn(*a)
    except Exception as e:  # noqa: BLE001
        return {"error": repr(e)[:200]}


def prefill_roofline(cfg, B, S, seconds):
    """Tensor roofline of one prefill (per GPU): algorithmic FLOPs = 2 B S x
    (every weight element, the tied LM head counted with the embedding) + per
    layer 2 x 2 B nq hd x (S^2 / 2 causal, or S W inside a window), against
    the measured burst bf16 GEMM peak."""
    from cljxla_b200.host import drivers as d
    params = sum(int(np.prod(shp)) for _, shp, _ in d.weight_specs(cfg))
    flops = 2.0 * B * S * params
    for i in range(cfg.layers):
        span = S * min(S, cfg.window) if cfg.is_local(i) else S * S / 2
        flops += 4.0 * B * cfg.n_heads * cfg.head_dim * span
    _, tc_peak, src = load_peaks()
    tf = flops / seconds / 1e12
    return {"bound": "tensor", "achieved": round(tf, 1), "peak": tc_peak, "unit": "TFLOP/s",
            "frac": round(tf / tc_peak, 4), "flops": round(flops), "peak_source": src + " (burst)"}


# DRAM traffic per launch of the dominant kernel class, from one ncu capture
# of the same kernels (dram__bytes_read.sum + dram__bytes_write.sum; the
# command and per-launch table are in profiles/gemv_bulk_copy_gemma3-4b_decode.md):
# the mean over a step's gemv_fused launches, 34 q/k/v, 34 gate/up and the LM head
NCU_TRAFFIC = {
    ("gemma3-4b decode, batch 1, prompt 2048, KV cache 2560 positions", "gemv_fused"): 81685995,
}


def ncu_traffic(workload, kind, dk):
    """The roofline's `traffic` (bytes per launch, from the ncu capture) beside
    the algorithmic bytes per launch it compares with; null for a workload or
    kernel class without a capture."""
    t = NCU_TRAFFIC.get((workload, kind))
    algo = dk["bytes"] / dk["calls"] if dk.get("calls") else None
    return {"traffic": t, "algorithmic_bytes_per_launch": round(algo) if algo else None,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, mean per launch"
                              if t else None}


def cpu_baseline(cfg, B, S, T, txt_dec, host_w, steps):
    """Times the numpy oracle on the same decode graph (all host threads)."""
    try:
        import psutil
        need = sum(w.size for w in host_w) * 4 * 1.3
        if psutil.virtual_memory().available < need:
            return {"value": None, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                    "sample": f"skipped: host RAM below {need / 1e9:.0f} GB needed for f32 weights"}
    except Exception:
        pass
    sys.path.insert(0, ROOT)
    from oracle import interp
    from cljxla_b200.host import drivers as d
    wf = [interp.bf16_bits_to_f32(w) if w.dtype == np.uint16 else w for w in host_w]
    kv = [np.zeros(d.cache_shape(cfg, B, T), np.float32) for _ in range(2 * cfg.layers)]
    it = interp.Interpreter(txt_dec)
    x = np.zeros((B, 1), np.int32)
    t0 = time.perf_counter()
    for i in range(max(1, steps)):
        it.run([x, d.pos_inputs(cfg, "decode", B, S + i, 1)] + wf + kv)
    dt = (time.perf_counter() - t0) / max(1, steps)
    return {"value": B / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{max(1, steps)} decode step(s) of the same graph at position {S}, numpy oracle "
                      f"(CPU restatement of the reference graph, not the reference binary), {dt:.2f} s/step"}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.tp > 1 and args.tp != world:
        raise SystemExit(f"--tp {args.tp} needs exactly {args.tp} ranks (torchrun --nproc-per-node {args.tp})")
    import torch
    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    cfg, B, S, T, res = run_ours(args, rank, world, local_rank)
    if res is None:
        return
    if world > 1:
        t = torch.tensor([res["dec_s"], res["e2e_s"], res["prefill_s"]], device=f"cuda:{local_rank}")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dec_s, e2e_s, pre_s = [float(x) for x in t.tolist()]
    else:
        dec_s, e2e_s, pre_s = res["dec_s"], res["e2e_s"], res["prefill_s"]
    tp = None
    if not args.no_tp_block and args.tp == 1 and not args.tiny and not args.layers and world in (1, 2, 4, 8):
        try:
            tp = tp_block(args, rank, world, local_rank)
        except Exception as e:  # noqa: BLE001 - the data-parallel line stands; the block says what failed
            tp = {"error": repr(e)[:300]}
    if rank == 0:
        replicas = world // max(1, args.tp)
        value = replicas * res["tokens"] / dec_s
        dk = res["by_kind"][res["dom"]]
        wl = (f"{args.config} decode, batch {B}, prompt {S}, KV cache {T} positions"
              + (" [tiny]" if args.tiny else "") + (f" [{args.layers} layers]" if args.layers else ""))
        line = {
            "metric": "decode tokens/s (greedy KV-cached decode step, whole job)",
            "value": round(value, 2),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dec_s / args.steps * 1e3, 4),
            "higher_is_better": True,
            "scaling": "weak" if args.tp == 1 else "strong",
            "vs_baseline": None,
            "dtype": cfg.dtype,
            "data": "synthetic (random-init weights N(0,0.02), random token ids)",
            "config": {"workload": wl,
                       "model": args.config, "global_batch": B * replicas, "seq_len": S, "kv_len": T,
                       "parallelism": (f"dp{world} (independent replicas)" if args.tp == 1 else
                                       f"tp{args.tp}" + (f" x dp{replicas}" if replicas > 1 else "")
                                       + " (NCCL all-reduce after attention and MLP)"),
                       "l2": "weights stream >> 126 MB L2 every step (no flush needed)"},
            "prefill": {"value": round(replicas * B * S / pre_s, 1), "unit": "tokens/s",
                        "ms": round(pre_s * 1e3, 3), "graph": "dynamic-position prefill",
                        "roofline": safe(prefill_roofline, cfg, B, S, pre_s),
                        "kernel_time_by_kind_ms": res["pre_by_kind"]},
            "e2e": ({"value": round(replicas * res["e2e_tokens"] / e2e_s, 2), "unit": "tokens/s",
                     "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 4 * B,
                     "path": "PJRT C ABI: BufferFromHostBuffer (token, position), Execute of the decode graph "
                             "with in-graph greedy argmax (tensor.clj:519-532), ToHostBuffer of the token ids",
                     "logits_path": {"value": round(replicas * res["e2e_tokens"] / res["e2e_logits_s"], 2),
                                     "d2h_bytes_per_step": res["logits_bytes"],
                                     "path": "decode graph returning f32 logits + host argmax (argmax-host)"}}
                    if res["e2e_greedy"] else
                    {"value": round(replicas * res["e2e_tokens"] / e2e_s, 2), "unit": "tokens/s",
                     "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": res["logits_bytes"],
                     "path": "PJRT C ABI (BufferFromHostBuffer, Execute, ToHostBuffer) + host argmax"}),
            "roofline": {"bound": "hbm", "kernel": res["dom"],
                         "achieved": round(res["achieved"], 1), "peak": res["hbm_peak"], "unit": "GB/s",
                         "frac": round(res["achieved"] / res["hbm_peak"], 4),
                         **ncu_traffic(wl, res["dom"], dk),
                         "peak_source": res["peak_src"],
                         "share_of_step": round(dk["ms"] / res["total_ms"], 4) if res["total_ms"] else None},
            "cpu_baseline": res["cpu"],
            "clocks": res["clocks"],
            "gpu_launches": res["launches"],
            "kernel_time_by_kind_ms": {k: round(v["ms"] / 2, 4) for k, v in res["by_kind"].items()},
            "plan": res["plan"],
        }
        if tp is not None:
            line["tp"] = tp
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_reference(args, rank, world):
    """CPU restatement of the reference path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    sys.path.insert(0, ROOT)
    _pkg()
    from oracle import interp
    from cljxla_b200.host import drivers as d
    from cljxla_b200.host import stablehlo as shlo
    cfg, B, S, T = model_setup(args)
    # the same global batch as the repo arm at this N (one sequence batch per
    # data-parallel replica), decoded by the one CPU process
    B = B * max(1, world // max(1, args.tp))
    rng = np.random.Generator(np.random.PCG64(1234))
    wf = []
    for name, shp, kind in d.weight_specs(cfg):
        if kind == "mat":
            a = rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        elif kind == "plain_norm":
            a = np.float32(1) + rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        elif kind == "gemma_norm":
            a = rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        elif kind == "one":
            a = np.ones(shp, np.float32)
        else:
            a = np.zeros(shp, np.float32)
        wf.append(interp.round_bf16(a) if cfg.dtype == "bf16" else a)
    txt = shlo.graph_to_mlir_text(d.build_graph(cfg, "decode", B, S, T))
    it = interp.Interpreter(txt)
    kv = [np.zeros(d.cache_shape(cfg, B, T), np.float32) for _ in range(2 * cfg.layers)]
    x = np.zeros((B, 1), np.int32)
    for i in range(args.warmup):
        it.run([x, d.pos_inputs(cfg, "decode", B, S + i, 1)] + wf + kv)
    t0 = time.perf_counter()
    for i in range(args.steps):
        outs = it.run([x, d.pos_inputs(cfg, "decode", B, S + i, 1)] + wf + kv)
        kv = outs[1:]
    dt = time.perf_counter() - t0
    v = B * args.steps / dt
    line = {"impl": "reference", "metric": "decode tokens/s (greedy KV-cached decode step, whole job)",
            "value": round(v, 4), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": cfg.dtype, "data": "synthetic",
            "config": {"workload": f"{args.config} decode, batch {B}, prompt {S}, KV cache {T} positions",
                       "model": args.config, "global_batch": B, "seq_len": S},
            "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": "full decode steps of the printed graph on the numpy oracle (CPU "
                                       "restatement; the reference's JVM + xla_cpu_pjrt path is not installable here)"},
            "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
