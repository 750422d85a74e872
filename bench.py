#!/usr/bin/env python
"""Benchmark of the EXL3 MoE decode path on B200 (one JSON line on rank 0).

Workload (the metric's "MoE-layer decode"): Qwen-Next-like MoE decode, hidden 2048, 512 routed
experts of intermediate 512, top-10 softmax router (renormalised), K = 3 bits per weight, 48 layers, 4 tokens per
GPU. A step is one decode step of the batch through all 48 MoE layers: router -> prepare (alignment + rotated
activation rows) -> gate|up GEMV -> down GEMV -> fixed-order combine per layer, captured once in a CUDA graph and
replayed. With N GPUs the experts are sharded expert-parallel
(512/N per GPU) and tokens are data-parallel (4 per GPU): NCCL all-to-all dispatch/combine per layer.
Synthetic data: uniform random trellis bitstreams, +-1 sign vectors, activations ~N(0,1) fp16, router logits
~N(0,1) fp32, all seeded; weights are created on the device.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--workload qwen_next_decode|glm_decode]
"""
from __future__ import annotations

import argparse
import json
import math
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "b70-inference_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

WORKLOADS = {
    # BASELINE config 4
    "qwen_next_decode": dict(H=2048, E=512, I=512, topk=10, Ks=(3,), layers=48, router="softmax", batch=4,
                             act_limit=0.0, shared_K=0, res_frac=0.0, scale=1.0),
    # BASELINE config 3 (one GLM-like layer, repeated 8 times so that a step's weights exceed L2)
    "glm_decode": dict(H=6144, E=160, I=1536, topk=8, Ks=(2, 3), layers=8, router="sigmoid", batch=1,
                       act_limit=10.0, shared_K=4, res_frac=0.25, scale=2.5),
    # BASELINE config 5 (DeepSeek-V4-like MoE prefill, one layer per step): 8192 tokens, K in {1, 2} per projection
    # with P(K = 2) = 0.62 (1.62 bits average), shared expert K = 2, sqrt-softplus router, bf16 activations
    "dsv4_prefill": dict(H=7168, E=256, I=2048, topk=8, Ks=(1, 2), p_k2=0.62, layers=1, router="sqrt_softplus",
                         batch=8192, act_limit=10.0, shared_K=2, res_frac=0.0, scale=2.5, prefill=True),
}
METRIC = "MoE-layer decode tok/s + compressed-weight HBM GB/s (% of peak)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------------ CPU baseline

def _oracle_pick(args):
    """One (token, expert) evaluation of the oracle's expert math on host cores (worker process)."""
    import numpy as np
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    x, mats, act_limit = args
    ex = O.ExpertW(*mats)
    return O.expert_forward(x, ex, act_limit)


def _pick_tasks(cfg, rng, n_picks: int):
    """n_picks (token, expert) evaluations of the workload's shapes with fresh random weights (numpy)."""
    import numpy as np
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    H, I = cfg["H"], cfg["I"]
    tasks = []
    for _ in range(n_picks):
        x = rng.standard_normal((1, H)).astype(np.float16)
        K = int(rng.choice(cfg["Ks"]))
        mats = [(O.random_trellis(rng, kk, nn, K), O.random_signs(rng, kk), O.random_signs(rng, nn), K)
                for kk, nn in ((H, I), (H, I), (I, H))]
        tasks.append((x, mats, cfg["act_limit"]))
    return tasks


def cpu_picks_seconds(cfg, pool, rng, n_picks: int) -> float:
    """Wall seconds for the oracle port to evaluate n_picks expert picks in parallel over the pool's host cores."""
    import numpy as np
    tasks = _pick_tasks(cfg, rng, n_picks)
    t0 = time.perf_counter()
    outs = pool.map(_oracle_pick, tasks, chunksize=1)
    t = time.perf_counter() - t0
    assert all(np.isfinite(o).all() for o in outs)
    return t


def cpu_tok_s(cfg, picks: int, seconds: float) -> float:
    """tok/s of the full layer stack implied by `picks` expert evaluations taking `seconds`."""
    return (picks / cfg["topk"]) / (seconds * cfg["layers"])


def run_reference(args, cfg):
    """--impl reference: the reference's CPU algorithm (the oracle port of its torch path) on the host cores.
    Each step evaluates a bounded sample of the workload's expert picks in parallel on all host cores; the sample
    per step is sized so that the K timed steps take about two minutes at most."""
    import numpy as np
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(1234)
    with mp.get_context("spawn").Pool(cores) as pool:
        t1 = cpu_picks_seconds(cfg, pool, rng, cores)              # warm-up + sizing
        for _ in range(max(0, args.warmup - 1)):
            cpu_picks_seconds(cfg, pool, rng, cores)
        per_pick = t1 / max(1, math.ceil(cores / cores))
        picks = cores if per_pick * args.steps <= 120 else max(1, int(cores * 120 / (per_pick * args.steps)))
        ts = [cpu_picks_seconds(cfg, pool, rng, picks) for _ in range(args.steps)]
    t = statistics.median(ts)
    tok_s = cpu_tok_s(cfg, picks, t)
    ms_step = 1e3 / tok_s * cfg["batch"]
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": config_of(args, cfg),
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"{picks} expert picks per step (trellis decoded and applied per call, as the "
                                   f"reference's torch path does) in parallel on {cores} spawn workers; tok/s = "
                                   f"picks/topk/(step time x {cfg['layers']} layers)"},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_of(args, cfg):
    N = args.gpus
    return {"workload": args.workload, "hidden": cfg["H"], "experts": cfg["E"], "intermediate": cfg["I"],
            "topk": cfg["topk"], "K": list(cfg["Ks"]), "layers": cfg["layers"], "router": cfg["router"],
            "batch_per_gpu": cfg["batch"], "global_batch": cfg["batch"] * N,
            "parallelism": f"ep{N}" if N > 1 else "single",
            "l2": l2_note(cfg)}


def l2_note(cfg) -> str:
    """Whether a step's weight reads exceed the 126 MB L2 (picked experts of every layer; upper bound: all picks
    distinct)."""
    per_expert = 3 * cfg["H"] * cfg["I"] * max(cfg["Ks"]) / 8
    picks = min(cfg["E"], cfg["batch"] * cfg["topk"]) + (1 if cfg["shared_K"] else 0)
    lo = min(cfg["Ks"]) / max(cfg["Ks"]) * per_expert * min(cfg["E"], cfg["topk"]) * cfg["layers"]
    if lo > 126e6:
        return (f"inputs larger than L2: each step reads every layer's picked experts "
                f"(>= {lo / 1e9:.2f} GB of weights per step)")
    return f"inputs may fit in L2 ({per_expert * picks * cfg['layers'] / 1e6:.0f} MB of weights per step at most)"


# ------------------------------------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples during the timed region (clock, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        mhz, mx, reasons = [], None, set()
        for ln in self.lines:
            p = [v.strip() for v in ln.split(",")]
            if len(p) < 8:
                continue
            try:
                mhz.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ------------------------------------------------------------------------------------------------ ours

def build_layer(cfg, E_local, e_base, gen, dev):
    """One layer's local experts: gate/up/down trellis in three contiguous buffers, +-1 sign vectors."""
    import torch
    from exl3_b200 import moe
    H, I = cfg["H"], cfg["I"]
    Ks = cfg["Ks"]
    experts = []
    for e in range(E_local):
        K = Ks[(e_base + e) % len(Ks)] if len(Ks) > 1 else Ks[0]
        mats = []
        for kk, nn in ((H, I), (H, I), (I, H)):
            tr = torch.randint(-32768, 32767, (kk // 16, nn // 16, 16 * K), dtype=torch.int16, device=dev,
                               generator=gen)
            s1 = (torch.randint(0, 2, (kk,), device=dev, generator=gen) * 2 - 1).half()
            s2 = (torch.randint(0, 2, (nn,), device=dev, generator=gen) * 2 - 1).half()
            mats.append(moe.Exl3Matrix(tr, s1, s2, K))
        experts.append(moe.Expert(*mats))
    shared = None
    if cfg["shared_K"]:
        K = cfg["shared_K"]
        mats = []
        for kk, nn in ((H, I), (H, I), (I, H)):
            tr = torch.randint(-32768, 32767, (kk // 16, nn // 16, 16 * K), dtype=torch.int16, device=dev,
                               generator=gen)
            s1 = (torch.randint(0, 2, (kk,), device=dev, generator=gen) * 2 - 1).half()
            s2 = (torch.randint(0, 2, (nn,), device=dev, generator=gen) * 2 - 1).half()
            mats.append(moe.Exl3Matrix(tr, s1, s2, K))
        shared = moe.Expert(*mats)
    return moe.ExpertTable(experts, shared)


def run_prefill(args, cfg):
    """One MoE prefill layer per step (route + exl3_moe_prefill) timed with CUDA events over K steps. N > 1:
    expert parallelism (weak scaling): every rank routes its own `batch` tokens, holds E/N of the routed experts
    (plus the shared expert) and exchanges token rows with the others through ExpertParallelMoE (NCCL all-to-all
    dispatch and combine, the tcgen05 prefill kernels locally); value = all ranks' tokens / the slowest rank's step.
    roofline: tensor-bound; achieved = one rank's algorithmic flops (2 tokens topk 3 H I + shared 2 tokens 3 H I)
    / the step time (router, alignment, rotations, combine and the exchange included)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from exl3_b200 import _lib as L
    from exl3_b200 import ep, moe, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    cores = os.cpu_count() or 1
    pool = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        pool = mp.get_context("spawn").Pool(cores)          # started before the first CUDA call
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    H, E, I, topk, T = cfg["H"], cfg["E"], cfg["I"], cfg["topk"], cfg["batch"]
    E_local = E // world
    e0 = rank * E_local
    gen = torch.Generator(device=dev).manual_seed(11 + rank)

    def mat(k, n, K):
        tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=dev, generator=gen)
        s1 = (torch.randint(0, 2, (k,), device=dev, generator=gen) * 2 - 1).half()
        s2 = (torch.randint(0, 2, (n,), device=dev, generator=gen) * 2 - 1).half()
        return moe.Exl3Matrix(tr, s1, s2, K)

    experts = []
    for e in range(e0, e0 + E_local):
        rng = np.random.default_rng(1000 + e)               # the expert's bit widths do not depend on the rank count
        Ks = [2 if rng.random() < cfg["p_k2"] else 1 for _ in range(3)]
        experts.append(moe.Expert(mat(H, I, Ks[0]), mat(H, I, Ks[1]), mat(I, H, Ks[2])))
    shared = moe.Expert(mat(H, I, cfg["shared_K"]), mat(H, I, cfg["shared_K"]), mat(I, H, cfg["shared_K"]))
    table = moe.ExpertTable(experts, shared)
    del experts, shared
    x = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
    logits = torch.randn(T, E, device=dev, generator=gen)
    ggen = torch.Generator(device=dev).manual_seed(7)       # router bias shared by all ranks
    bias = torch.randn(E, device=dev, generator=ggen) * 0.1
    out = torch.empty(T, H, device=dev, dtype=torch.float32)
    ws = None
    epm = None
    if world == 1:
        need = L.lib().exl3_moe_prefill_workspace_size(T, topk, E, H, I, 1)
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
    else:
        epm = ep.ExpertParallelMoE(E, H, topk, None, table, cfg["act_limit"])

    def step():
        ids, w, _ = ops.route(logits, L.ROUTE_SQRT_SOFTPLUS, topk, bias=bias, scale=cfg["scale"])
        if world == 1:
            moe.moe_prefill(x, ids, w, table, cfg["act_limit"], out=out, workspace=ws)
        else:
            out.copy_(epm.forward(x, ids, w))

    def timed(body):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            body()
        t1.record()
        torch.cuda.synchronize()
        ms_ = t0.elapsed_time(t1) / args.steps
        if world > 1:
            tt = torch.tensor([ms_], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms_ = float(tt.item())
        return ms_

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms = timed(step)
    assert torch.isfinite(out).all(), "non-finite MoE output"
    assert L.lib().exl3_device_status(local) == 0

    # e2e: the same step from pinned host buffers (x, router logits) to a host output, copies inside the timed region
    xh, lh = x.cpu().pin_memory(), logits.cpu().pin_memory()
    oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e_step():
        x.copy_(xh, non_blocking=True)
        logits.copy_(lh, non_blocking=True)
        step()
        oh.copy_(out, non_blocking=True)

    ms_e2e = timed(e2e_step)
    assert torch.isfinite(oh).all(), "non-finite MoE output"

    cpu = None
    if pool is not None:
        rng2 = np.random.default_rng(5)
        cpu_picks_seconds(cfg, pool, rng2, cores)
        tcpu = statistics.median(cpu_picks_seconds(cfg, pool, rng2, cores) for _ in range(3))
        pool.close()
        cpu = {"value": round(cores / topk / tcpu, 5), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"{cores} expert picks of this layer (trellis decoded and applied per call) in parallel on "
                         f"{cores} spawn workers, median of 3; tok/s = picks/topk/time; numpy restatement of the "
                         f"reference's torch path"}
    flops = 2.0 * T * topk * 3 * H * I + 2.0 * T * 3 * H * I
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        peak = float(json.load(f)["bf16_tflops"])
    ach = flops / (ms * 1e-3) / 1e12
    # route, alignment (count + place when the pairs exceed one CTA's segment), rotation, gate and up GEMM,
    # activation, down GEMM, combine; N > 1: the local step on the received rows and the shared expert's own call
    per_call = lambda rows: 8 if rows * topk > 8192 else 7
    launches = (per_call(T) if world == 1 else 1 + per_call(T * world) + per_call(T)) * args.steps
    if rank == 0:
        line = {
            "metric": "MoE-layer prefill tok/s (tcgen05 grouped GEMM, tensor-pipe fraction)",
            "value": round(world * T / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random trellis, +-1 signs, N(0,1) bf16 activations)",
            "config": {"workload": args.workload, "tokens_per_gpu": T, "hidden": H, "experts": E,
                       "intermediate": I, "topk": topk, "K": "1/2 (P(2)=0.62)", "shared_K": cfg["shared_K"],
                       "router": cfg["router"], "parallelism": f"ep{world}" if world > 1 else "none",
                       "l2": "inputs larger than L2 (expert weights of 2.3 GB per 256 experts, 117 MB of activations "
                             "per rank and step)"},
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(ach / peak, 4), "peak_kind": "measured bf16 burst", "traffic": None,
                         "flops_per_step_per_gpu": flops},
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * T / (ms_e2e * 1e-3), 1), "unit": "tok/s",
                    "h2d_bytes_per_step": int(xh.numel() * 2 + lh.numel() * 4),
                    "d2h_bytes_per_step": int(oh.numel() * 4)},
            "gpu_launches": launches, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ours(args, cfg):
    import numpy as np
    import torch
    import torch.distributed as dist

    from exl3_b200 import _lib as L
    from exl3_b200 import ep, moe, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    cores = os.cpu_count() or 1
    pool = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        pool = mp.get_context("spawn").Pool(cores)          # started before the first CUDA call
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    H, E, I, topk, Ltot, B = cfg["H"], cfg["E"], cfg["I"], cfg["topk"], cfg["layers"], cfg["batch"]
    E_local = E // world
    e0 = rank * E_local
    kind = {"softmax": L.ROUTE_SOFTMAX, "sigmoid": L.ROUTE_SIGMOID, "sqrt_softplus": L.ROUTE_SQRT_SOFTPLUS}[
        cfg["router"]]
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    tables = [build_layer(cfg, E_local, e0, gen, dev) for _ in range(Ltot)]
    ggen = torch.Generator(device=dev).manual_seed(7)                  # router state shared by all ranks
    bias = (torch.randn(Ltot, E, device=dev, generator=ggen) * 0.1) if cfg["router"] != "softmax" else None
    res = None
    if cfg["res_frac"] > 0:
        res = torch.where(torch.rand(Ltot, E, device=dev, generator=ggen) < cfg["res_frac"], 0.1, 0.0).float()
    tgen = torch.Generator(device=dev).manual_seed(99 + rank)          # tokens differ per rank
    x = torch.randn(Ltot, B, H, device=dev, generator=tgen).half()
    logits = torch.randn(Ltot, B, E, device=dev, generator=tgen).float()
    out = torch.empty(Ltot, B, H, device=dev, dtype=torch.float32)
    epm = [ep.ExpertParallelMoE(E, H, topk, None, tables[l], cfg["act_limit"]) for l in range(Ltot)] if world > 1 \
        else None
    ev_pairs = {}

    def step(events=None):
        for l in range(Ltot):
            ids, w, _ = ops.route(logits[l], kind, topk, bias=None if bias is None else bias[l],
                                  res=None if res is None else res[l], scale=cfg["scale"], renorm=True)
            if world == 1:
                moe.moe_forward(x[l], ids, w, tables[l], cfg["act_limit"], torch.float32, out=out[l], events=events)
            else:
                out[l].copy_(epm[l].forward(x[l], ids, w))

    # eager warm-up (first calls configure kernel attributes, NCCL communicators)
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # capture one decode step twice: as the timed graph, and with external event nodes around each GEMV launch
    # (event nodes between kernels end the programmatic overlap of neighbouring launches, so that copy is replayed
    # only after the timed region, to measure the gate|up kernel's own duration)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()                                                          # warm the side stream
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    ev = {"external": True} if world == 1 else None
    graph_ev = None
    if ev is not None:
        graph_ev = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_ev):
            step(ev)
    # ---- timed: K replays of the captured step, inputs resident in HBM (clocks sampled from the warm-up on) ----
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0.record()
        for _ in range(args.steps):
            graph.replay()
        t1.record()
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
        dist.barrier()
    tok_s = B * world / (ms * 1e-3)
    if graph_ev is not None:
        for _ in range(3):
            graph_ev.replay()
        torch.cuda.synchronize()

    # ---- dominant kernel (gate|up GEMV): durations from the event nodes of the last replay ----
    gu_ms = None
    if ev is not None and ev.get("gateup"):
        gu = [a.elapsed_time(b) for a, b in ev["gateup"]]
        gu_ms = sum(gu) / len(gu)

    # ---- algorithmic bytes: experts picked in each layer (routing is fixed across steps) ----
    gu_bytes = 0
    w_bytes = 0
    for l in range(Ltot):
        ids, _, _ = ops.route(logits[l], kind, topk, bias=None if bias is None else bias[l],
                              res=None if res is None else res[l], scale=cfg["scale"], renorm=True)
        t = tables[l]
        uniq = sorted({int(e) for e in ids.reshape(-1).tolist() if e0 <= e < e0 + E_local})
        if world > 1:
            allid = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(allid, ids)
            uniq = sorted({int(e) - e0 for a in allid for e in a.reshape(-1).tolist() if e0 <= e < e0 + E_local})
        else:
            uniq = [e - e0 for e in uniq]
        exs = [t.experts[e] for e in uniq] + ([t.shared] if t.shared is not None else [])
        for ex in exs:
            for m in (ex.gate, ex.up):
                b = m.trellis.numel() * 2 + (m.k + m.n) * 2
                gu_bytes += b
                w_bytes += b
            w_bytes += ex.down.trellis.numel() * 2 + (ex.down.k + ex.down.n) * 2
        npairs = B * topk + (B if t.shared is not None else 0)
        gu_bytes += B * H * 2 + npairs * I * 2
    peak, peak_kind = peaks()
    roof = None
    if gu_ms:
        ach = gu_bytes / Ltot / (gu_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": TRAFFIC_PER_LAUNCH.get(args.workload), "kernel": "k_gemv<EPI_GATEUP> (gate|up GEMV)",
                "peak_kind": peak_kind, "launch_ms": round(gu_ms, 5), "bytes_per_launch": gu_bytes // Ltot}
    weight_gbs = w_bytes * world / (ms * 1e-3) / 1e9 if world == 1 else None
    if world > 1:
        wb = torch.tensor([float(w_bytes)], device=dev)
        dist.all_reduce(wb)
        weight_gbs = float(wb.item()) / (ms * 1e-3) / 1e9

    # ---- e2e: the same step with host buffers (pinned), copies inside the timed region ----
    xh = x.cpu().pin_memory()
    lh = logits.cpu().pin_memory()
    oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    e0_, e1_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0_.record()
    for _ in range(args.steps):
        x.copy_(xh, non_blocking=True)
        logits.copy_(lh, non_blocking=True)
        graph.replay()
        oh.copy_(out, non_blocking=True)
    e1_.record()
    torch.cuda.synchronize()
    ms_e2e = e0_.elapsed_time(e1_) / args.steps
    if world > 1:
        tt = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_e2e = float(tt.item())
    assert torch.isfinite(oh).all(), "non-finite MoE output"
    status = L.lib().exl3_device_status(0)
    assert status == 0, f"device status {status}"

    cpu = None
    if pool is not None:
        rng = np.random.default_rng(5)
        cpu_picks_seconds(cfg, pool, rng, cores)
        t = statistics.median(cpu_picks_seconds(cfg, pool, rng, cores) for _ in range(3))
        pool.close()
        cpu = {"value": round(cpu_tok_s(cfg, cores, t), 4), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"{cores} expert picks (trellis decoded and applied per call) in parallel on {cores} spawn "
                         f"workers, median of 3; tok/s = picks/topk/(time x {Ltot} layers); numpy restatement of "
                         f"the reference's torch path"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded random trellis, +-1 signs, N(0,1))",
            "config": config_of(args, cfg),
            "weight_gbs": round(weight_gbs, 1), "weight_gbs_frac": round(weight_gbs / world / peak, 4),
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(B * world / (ms_e2e * 1e-3), 2), "unit": "tok/s",
                    "h2d_bytes_per_step": int(xh.numel() * 2 + lh.numel() * 4),
                    "d2h_bytes_per_step": int(oh.numel() * 4)},
            "gpu_launches": 5 * Ltot * args.steps,          # route, prepare, gate|up, down, combine per layer
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    del graph, graph_ev
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# DRAM bytes (read + write) per gate|up launch from the committed ncu capture
# (profiles/k_gemv_moe_qwen_next_full.md), per workload; None where no capture was made.
TRAFFIC_PER_LAUNCH: dict = {"qwen_next_decode": 31216384 + 39680}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qwen_next_decode", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=0, help="tokens per GPU (default: the workload's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (small profiling captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    cfg = dict(WORKLOADS[args.workload])
    if args.batch:
        cfg["batch"] = args.batch
    if args.layers:
        cfg["layers"] = args.layers
    if args.impl == "reference":
        run_reference(args, cfg)
    elif cfg.get("prefill"):
        run_prefill(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
