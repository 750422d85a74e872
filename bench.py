#!/usr/bin/env python
"""Benchmark of the EXL3 trellis path on B200 (one JSON line on rank 0).

Primary workload (the metric's "MoE-layer decode"): Qwen-Next-like MoE decode, hidden 2048, 512
routed experts of intermediate 512, top-10 softmax router (renormalised), K = 3 bits per weight, 48 layers, 4 tokens
per GPU. A step is one decode step of the batch through all 48 MoE layers: router -> prepare (alignment + rotated
activation rows) -> gate|up GEMV -> down GEMV -> fixed-order combine per layer, captured once in a CUDA graph and
replayed. With N GPUs the experts are sharded expert-parallel (512/N per GPU), tokens are data-parallel (4 per GPU)
and the peer-memory exchange kernels (dispatch / combine / reduce over NVLink) move the routed rows; before timing, an extra layer held in full by every rank
checks that the expert-parallel output equals the local one (exit 1 on a mismatch, before any line is printed).

The same line carries the other BASELINE configurations under "extra" (default run only; --workload runs one alone):
  glm_decode    config 3: GLM-like MoE decode layer (H 6144, 160 experts + shared K 4, I 1536, K 2/3, top-8 sigmoid,
                +0.1 on a resident 25 %), 8 layers per step so that a step's weights exceed L2, batch 1 per GPU;
  dsv4_prefill  config 5: DeepSeek-V4-like MoE prefill (8192 tokens per GPU, H 7168, 256 experts + shared, I 2048,
                K 1/2 with P(2) = 0.62, top-8 sqrt-softplus), tcgen05 grouped GEMMs, expert-parallel for N > 1;
  dense_decode  config 2: a 60-layer stack of EXL3 linears 5120->25600, 25600->5120, 5120->5120 at K 2/3/4/5 and
                batch 1/2/4 (replicas for N > 1), the stack replayed in one CUDA graph.
Synthetic data: uniform random trellis bitstreams, +-1 sign vectors, activations ~N(0,1), router logits ~N(0,1)
fp32, all seeded; weights are created on the device (no checkpoints exist here).

cpu_baseline / --impl reference: the reference's algorithm for the path (the oracle port of its torch CPU code:
trellis decoded per call, then applied) on the host cores, one single-threaded worker process per core, timed as
measured wall time of real work (see run_reference).

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--workload NAME] [--no-extra]
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
    "qwen_next_decode": dict(kind="decode", H=2048, E=512, I=512, topk=10, Ks=(3,), layers=48, router="softmax",
                             batch=4, act_limit=0.0, shared_K=0, res_frac=0.0, scale=1.0, batch_sweep=(1, 2)),
    # BASELINE config 3 (one GLM-like layer shape, 8 layers per step so that a step's weights exceed L2)
    "glm_decode": dict(kind="decode", H=6144, E=160, I=1536, topk=8, Ks=(2, 3), layers=8, router="sigmoid", batch=1,
                       act_limit=10.0, shared_K=4, res_frac=0.25, scale=2.5),
    # K in {1, 2} per projection with P(K = 2) = 0.62 (1.62 bits average), shared expert K = 2
    "dsv4_prefill": dict(kind="prefill", H=7168, E=256, I=2048, topk=8, Ks=(1, 2), p_k2=0.62, layers=1,
                         router="sqrt_softplus", batch=8192, act_limit=10.0, shared_K=2, res_frac=0.0, scale=2.5),
    # BASELINE config 2 (and config 1 for the CPU timing): 60 layers x (5120->25600, 25600->5120, 5120->5120)
    "dense_decode": dict(kind="dense", shapes=((5120, 25600), (25600, 5120), (5120, 5120)), layers=60,
                         Ks=(2, 3, 4, 5), batches=(1, 2, 4)),
}
EXTRAS = ("glm_decode", "dsv4_prefill", "dense_decode")
EXTRA_MAX_STEPS = 50
METRIC = "MoE-layer decode tok/s + compressed-weight HBM GB/s (% of peak)"


def peaks():
    """(hbm GB/s, bf16 TFLOP/s burst, kind): the driver-measured peaks, else the recipe's fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------------------------------------------ CPU baseline

_BANK: dict = {}


def _cpu_task(task):
    """One unit of the reference's CPU work in a single-threaded worker: an expert pick (gate, up, down linears with
    the trellis decoded per call, as the reference's torch path does) or one dense linear. The expert's / linear's
    random weights are generated on first use and cached in the worker; the returned value is the elapsed time of
    the evaluation alone."""
    import numpy as np
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    kind, key, shape, seed = task
    if key not in _BANK:
        rng = np.random.default_rng(seed)
        if kind == "pick":
            H, I, Ks, act_limit = shape
            mats = [(O.random_trellis(rng, kk, nn, K), O.random_signs(rng, kk), O.random_signs(rng, nn), K)
                    for (kk, nn), K in zip(((H, I), (H, I), (I, H)), Ks)]
            _BANK[key] = (O.ExpertW(*mats), rng.standard_normal((1, H)).astype(np.float16), act_limit)
        else:
            k, n, K = shape
            _BANK[key] = ((O.random_trellis(rng, k, n, K), O.random_signs(rng, k), O.random_signs(rng, n), K),
                          rng.standard_normal((1, k)).astype(np.float16))
    t0 = time.perf_counter()
    if kind == "pick":
        ex, x, act_limit = _BANK[key]
        y = O.expert_forward(x, ex, act_limit)
    else:
        (tr, s1, s2, K), x = _BANK[key]
        y = O.exl3_linear(x, tr, s1, s2, K, np.float16)
    dt = time.perf_counter() - t0
    assert np.isfinite(y.astype(np.float32)).all()
    return dt


def cpu_pool(cores: int):
    """`cores` spawn workers, each limited to one BLAS / OpenMP thread (set in the environment they start with), so
    that the workers do not oversubscribe the host. Started before the first CUDA call."""
    keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS", "NUMEXPR_NUM_THREADS")
    old = {k: os.environ.get(k) for k in keys}
    for k in keys:
        os.environ[k] = "1"
    try:
        return mp.get_context("spawn").Pool(cores)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def pick_tasks(cfg, wl: str, n: int, first: int = 0):
    """n expert picks of the workload (bit widths as the GPU run draws them)."""
    tasks = []
    for i in range(first, first + n):
        if wl == "dsv4_prefill":
            import numpy as np
            rng = np.random.default_rng(1000 + i)
            Ks = tuple(2 if rng.random() < cfg["p_k2"] else 1 for _ in range(3))
        else:
            K = cfg["Ks"][i % len(cfg["Ks"])]
            Ks = (K, K, K)
        tasks.append(("pick", (wl, i), (cfg["H"], cfg["I"], Ks, cfg["act_limit"]), 7000 + i))
    return tasks


def timed_map(pool, tasks):
    """Wall seconds of evaluating the tasks in parallel on the pool (the step), and the sum of the evaluations'
    own times."""
    t0 = time.perf_counter()
    per = pool.map(_cpu_task, tasks, chunksize=1)
    return time.perf_counter() - t0, sum(per)


def cpu_decode_baseline(pool, cores, wl, cfg):
    """One layer of the decode batch per step: all its picks (+ the shared expert per token) in parallel; median of
    three measured steps after one warm-up step. tok/s = batch / (layer wall time x layers)."""
    B, topk = cfg["batch"], cfg["topk"]
    tasks = pick_tasks(cfg, wl, B * topk)
    if cfg["shared_K"]:
        sk = cfg["shared_K"]
        tasks += [("pick", (wl, "shared", t), (cfg["H"], cfg["I"], (sk, sk, sk), cfg["act_limit"]), 99 + t)
                  for t in range(B)]
    timed_map(pool, tasks)
    ts = [timed_map(pool, tasks)[0] for _ in range(3)]
    t = statistics.median(ts)
    return {"value": round(B / (t * cfg["layers"]), 5), "unit": "tok/s", "cores": cores, "kind": "port",
            "layer_ms": round(t * 1e3, 2), "cpu": cpu_model(),
            "sample": f"one whole layer per step: {len(tasks)} expert evaluations ({B} tokens x top-{topk}"
                      f"{' + shared' if cfg['shared_K'] else ''}; trellis decoded and applied per call) on {cores} "
                      f"single-threaded workers, median of 3 measured steps; tok/s = {B} tokens / (layer time x "
                      f"{cfg['layers']} layers)"}


def cpu_prefill_baseline(pool, cores, wl, cfg):
    """A bounded sample of the prefill layer's picks: one pick per worker (plus one shared-expert row), timed as
    one parallel step; tok/s = picks / topk / wall time (the layer has tokens x topk picks)."""
    tasks = pick_tasks(cfg, wl, cores)
    timed_map(pool, tasks)
    t, _ = timed_map(pool, tasks)
    return {"value": round(cores / cfg["topk"] / t, 5), "unit": "tok/s", "cores": cores, "kind": "port",
            "cpu": cpu_model(),
            "sample": f"{cores} expert picks of the layer (one per single-threaded worker; trellis decoded and applied "
                      f"per call) in one measured step of {t:.1f} s; tok/s = picks / topk / time"}


def cpu_dense_baseline(pool, cores, cfg):
    """BASELINE config 1 on the host: one EXL3 linear in = out = 4096, K = 4, x [1, 4096] (trellis decoded per call),
    one per worker in parallel; the stack's tok/s at K = 4, batch 1 follows from the measured rate of trellis
    bytes (the three config-2 shapes per layer, 60 layers)."""
    tasks = [("linear", ("cfg1", i), (4096, 4096, 4), 500 + i) for i in range(cores)]
    timed_map(pool, tasks)
    t, tsum = timed_map(pool, tasks)
    per_call = tsum / cores
    rate = cores * 4096 * 4096 * 4 / 8 / t                               # trellis bytes per second, all workers
    stack_bytes = cfg["layers"] * sum(k * n for k, n in cfg["shapes"]) * 4 / 8
    return {"value": round(rate / stack_bytes, 6), "unit": "tok/s", "cores": cores, "kind": "port",
            "cpu": cpu_model(), "config1_linear_ms": round(per_call * 1e3, 1),
            "sample": f"BASELINE config 1 (4096 x 4096, K 4, one row) once per single-threaded worker, {cores} in "
                      f"parallel ({per_call * 1e3:.0f} ms per call); tok/s of the 60-layer K 4 stack = measured "
                      f"trellis bytes per second / the stack's bytes"}


def run_reference(args, cfg):
    """--impl reference: the reference's CPU algorithm for the path (the oracle port of its torch code: trellis
    decoded per call, then applied) on the host cores, one single-threaded worker per core. A step evaluates a sample
    of one decode layer's expert picks in parallel: the whole layer (batch x top-k picks) when K such steps fit in
    about two minutes, else as many picks as do. value = tok/s of the 48-layer model implied by the measured step
    time: batch / (step time x picks per layer / picks per step x layers). ms_per_step = the measured step time."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if cfg["kind"] != "decode":
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the decode workloads"}))
        return
    cores = os.cpu_count() or 1
    pool = cpu_pool(cores)
    wl = args.workload
    B, topk = cfg["batch"], cfg["topk"]
    layer = pick_tasks(cfg, wl, B * topk)
    probe = layer[:cores]
    timed_map(pool, probe)                                               # warm the workers' caches
    t_probe, _ = timed_map(pool, probe)                                  # one parallel round of picks
    rounds_per_layer = math.ceil(len(layer) / cores)
    budget = 120.0 / max(1, args.steps + args.warmup)
    rounds = max(1, min(rounds_per_layer, int(budget / max(t_probe, 1e-6))))
    picks = min(len(layer), rounds * cores)
    sample = layer[:picks]
    for _ in range(max(0, args.warmup - 1)):
        timed_map(pool, sample)
    ts = [timed_map(pool, sample)[0] for _ in range(args.steps)]
    pool.close()
    t = statistics.median(ts)
    layer_s = t * len(layer) / picks
    tok_s = B / (layer_s * cfg["layers"])
    cpu = {"value": round(tok_s, 5), "unit": "tok/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
           "threads": f"{cores} worker processes x 1 thread",
           "sample": f"{picks} of the layer's {len(layer)} expert picks per step (trellis decoded and applied per "
                     f"call, as the reference's torch path does) on {cores} single-threaded workers; tok/s = {B} / "
                     f"(step time x {len(layer)}/{picks} x {cfg['layers']} layers)"}
    line = {
        "impl": "reference", "metric": METRIC, "value": cpu["value"], "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": config_of(args.workload, cfg, args.gpus), "layers_per_model_step": cfg["layers"],
        "picks_per_step": picks, "picks_per_layer": len(layer),
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_of(wl, cfg, N):
    if cfg["kind"] == "dense":
        return {"workload": wl, "shapes": [list(s) for s in cfg["shapes"]], "layers": cfg["layers"],
                "K": list(cfg["Ks"]), "batch": list(cfg["batches"]), "parallelism": f"replicas{N}" if N > 1 else
                "single", "l2": "inputs larger than L2 (the stack holds 4.3-10.8 GB of weights per K)"}
    c = {"workload": wl, "hidden": cfg["H"], "experts": cfg["E"], "intermediate": cfg["I"], "topk": cfg["topk"],
         "K": list(cfg["Ks"]), "layers": cfg["layers"], "router": cfg["router"], "batch_per_gpu": cfg["batch"],
         "global_batch": cfg["batch"] * N, "parallelism": f"ep{N}" if N > 1 else "single", "l2": l2_note(cfg)}
    if cfg.get("shared_K"):
        c["shared_K"] = cfg["shared_K"]
    if cfg.get("res_frac"):
        c["resident_frac_bias"] = [cfg["res_frac"], 0.1]
    return c


def l2_note(cfg) -> str:
    """Whether a step's weight reads exceed the 126 MB L2 (picked experts of every layer)."""
    per_expert = 3 * cfg["H"] * cfg["I"] * min(cfg["Ks"]) / 8
    lo = per_expert * min(cfg["E"], cfg["topk"]) * cfg["layers"]
    if cfg["kind"] == "prefill":
        return "inputs larger than L2 (every expert's weights, GBs, and the token rows each step)"
    return (f"inputs larger than L2: each step reads every layer's picked experts (>= {lo / 1e9:.2f} GB of weights "
            f"per step)" if lo > 126e6 else f"inputs may fit in L2 ({lo / 1e6:.0f} MB)")


# ------------------------------------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples (every 20 ms) while the timed region runs: SM clock, throttle reasons."""
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
                                          "-i", str(self.index), "-lms", "20"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.1)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.05)
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


# ------------------------------------------------------------------------------------------------ GPU context

class Ctx:
    """Process layout (RANK / LOCAL_RANK / WORLD_SIZE from torchrun), device, process group, CPU pool."""

    def __init__(self, args, want_pool: bool):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != args.gpus:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {self.world}")
        self.cores = os.cpu_count() or 1
        self.pool = cpu_pool(self.cores) if (want_pool and self.rank == 0 and self.world == 1) else None
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=self.dev)

    def max_over_ranks(self, v: float) -> float:
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return v
        t = torch.tensor([v], device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(self, v: float) -> float:
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return v
        t = torch.tensor([v], device=self.dev)
        dist.all_reduce(t)
        return float(t.item())

    def barrier(self):
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier()

    def close(self):
        import torch.distributed as dist
        if self.pool is not None:
            self.pool.close()
        if self.world > 1:
            dist.barrier()
            dist.destroy_process_group()


def rand_matrix(gen, dev, k, n, K, svh_scale=1.0):
    import torch
    from exl3_b200 import moe
    tr = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), dtype=torch.int16, device=dev, generator=gen)
    s1 = (torch.randint(0, 2, (k,), device=dev, generator=gen) * 2 - 1).half()
    s2 = ((torch.randint(0, 2, (n,), device=dev, generator=gen) * 2 - 1) * svh_scale).half()
    return moe.Exl3Matrix(tr, s1, s2, K)


def build_layer(cfg, E_local, e_base, gen, dev):
    """One decode layer's local experts (K per expert from the workload's list by global index) + shared expert."""
    from exl3_b200 import moe
    H, I, Ks = cfg["H"], cfg["I"], cfg["Ks"]
    experts = []
    for e in range(E_local):
        K = Ks[(e_base + e) % len(Ks)]
        experts.append(moe.Expert(rand_matrix(gen, dev, H, I, K), rand_matrix(gen, dev, H, I, K),
                                  rand_matrix(gen, dev, I, H, K)))
    shared = None
    if cfg["shared_K"]:
        K = cfg["shared_K"]
        shared = moe.Expert(rand_matrix(gen, dev, H, I, K), rand_matrix(gen, dev, H, I, K),
                            rand_matrix(gen, dev, I, H, K))
    return moe.ExpertTable(experts, shared)


def ep_check(ctx):
    """Expert-parallel correctness on the GPUs (N > 1): one small layer whose experts every rank holds in full.
    Each rank runs its own tokens through ExpertParallelMoE (its expert shard, peer-memory dispatch / combine) and through
    moe_forward on the full table; the two must agree within the parity tolerance (2e-3 relative, 1e-2 max-abs
    scaled to the output rms), at a decode batch (decode kernels) and at a prefill batch (tcgen05 kernels locally).
    Returns the worst relative error over ranks; raises SystemExit(1) on every rank if any rank mismatches."""
    import torch
    from exl3_b200 import _lib as L
    from exl3_b200 import ep, moe, ops
    W = ctx.world
    E, H, I, topk = 8 * W, 512, 256, 4
    gen = torch.Generator(device=ctx.dev).manual_seed(4242)              # identical experts on every rank
    full = [moe.Expert(rand_matrix(gen, ctx.dev, H, I, 2 + e % 3), rand_matrix(gen, ctx.dev, H, I, 3),
                       rand_matrix(gen, ctx.dev, I, H, 2 + (e + 1) % 3)) for e in range(E)]
    shared = moe.Expert(rand_matrix(gen, ctx.dev, H, I, 3), rand_matrix(gen, ctx.dev, H, I, 3),
                        rand_matrix(gen, ctx.dev, I, H, 3))
    e0, e1 = ep.expert_range(E, ctx.rank, W)
    local_tab = moe.ExpertTable(full[e0:e1], shared)
    full_tab = moe.ExpertTable(full, shared)
    worst = 0.0
    for B in (4, 700):
        tg = torch.Generator(device=ctx.dev).manual_seed(100 + ctx.rank)
        x = torch.randn((B, H), device=ctx.dev, generator=tg).half()
        logits = torch.randn((B, E), device=ctx.dev, generator=tg)
        ids, w, _ = ops.route(logits, L.ROUTE_SOFTMAX, topk)
        epm = ep.ExpertParallelMoE(E, H, topk, None, local_tab, 10.0)
        got = epm.forward(x, ids, w)
        fn = moe.moe_prefill if B * topk >= ep.PREFILL_MIN_PAIRS else moe.moe_forward
        ref = fn(x, ids, w, full_tab, 10.0)
        torch.cuda.synchronize()
        d = (got.double() - ref.double())
        rel = float(d.norm() / ref.double().norm().clamp_min(1e-30))
        mx = float(d.abs().max())
        rms = float(ref.double().pow(2).mean().sqrt())
        bad = not (rel <= 2e-3 and mx <= 1e-2 * max(1.0, rms) and torch.isfinite(got).all())
        worst = max(worst, rel)
        nbad = ctx.sum_over_ranks(1.0 if bad else 0.0)
        if nbad > 0:
            if ctx.rank == 0:
                print(f"expert-parallel check FAILED at batch {B}: {int(nbad)} rank(s) differ from the local result "
                      f"(rank 0: rel {rel:.3e}, max abs {mx:.3e})", file=sys.stderr, flush=True)
            raise SystemExit(1)
    return ctx.max_over_ranks(worst)


# ------------------------------------------------------------------------------------------------ decode

def run_decode(ctx, args, wl, cfg, steps, warmup, primary: bool):
    """MoE decode workload: a step = one decode step of the batch through the workload's layers, captured in a CUDA
    graph and replayed. roofline: the gate|up GEMV (k_gemv<EPI_GATEUP>), the step's dominant kernel, timed by
    external event nodes around each launch in a second captured copy of the step replayed after the timed region;
    algorithmic bytes = the picked experts' gate and up trellis + sign vectors + the activation rows it reads and
    writes."""
    import torch
    from exl3_b200 import _lib as L
    from exl3_b200 import ep, moe, ops
    world, rank = ctx.world, ctx.rank
    H, E, I, topk, Ltot, B = cfg["H"], cfg["E"], cfg["I"], cfg["topk"], cfg["layers"], cfg["batch"]
    E_local = E // world
    e0 = rank * E_local
    kind = {"softmax": L.ROUTE_SOFTMAX, "sigmoid": L.ROUTE_SIGMOID, "sqrt_softplus": L.ROUTE_SQRT_SOFTPLUS}[
        cfg["router"]]
    dev = ctx.dev
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
    epm = [ep.ExpertParallelMoE(E, H, topk, None, tables[l], cfg["act_limit"], capacity=B) for l in range(Ltot)] \
        if world > 1 else None

    def step(events=None):
        for l in range(Ltot):
            ids, w, _ = ops.route(logits[l], kind, topk, bias=None if bias is None else bias[l],
                                  res=None if res is None else res[l], scale=cfg["scale"], renorm=True)
            if world == 1:
                moe.moe_forward(x[l], ids, w, tables[l], cfg["act_limit"], torch.float32, out=out[l], events=events)
            else:
                epm[l].forward(x[l], ids, w, out=out[l])

    for _ in range(2):                                                  # eager: kernel attributes, communicators
        step()
    torch.cuda.synchronize()
    ctx.barrier()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
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
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(ctx.local) as clk:
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        ctx.barrier()
        t0.record()
        for _ in range(steps):
            graph.replay()
        t1.record()
        torch.cuda.synchronize()
    ms = ctx.max_over_ranks(t0.elapsed_time(t1) / steps)
    ctx.barrier()
    tok_s = B * world / (ms * 1e-3)
    gu_ms = None
    if graph_ev is not None:
        for _ in range(3):
            graph_ev.replay()
        torch.cuda.synchronize()
        gu = [a.elapsed_time(b) for a, b in ev["gateup"]]
        gu_ms = sum(gu) / len(gu)

    # algorithmic bytes: the experts picked in each layer (the routing is the same in every step)
    gu_bytes = w_bytes = 0
    import torch.distributed as dist
    for l in range(Ltot):
        ids, _, _ = ops.route(logits[l], kind, topk, bias=None if bias is None else bias[l],
                              res=None if res is None else res[l], scale=cfg["scale"], renorm=True)
        t = tables[l]
        if world > 1:
            allid = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(allid, ids)
            uniq = sorted({int(e) - e0 for a in allid for e in a.reshape(-1).tolist() if e0 <= e < e0 + E_local})
        else:
            uniq = sorted({int(e) for e in ids.reshape(-1).tolist() if 0 <= e < E})
        exs = [t.experts[e] for e in uniq] + ([t.shared] if t.shared is not None else [])
        for ex in exs:
            for m in (ex.gate, ex.up):
                b = m.trellis.numel() * 2 + (m.k + m.n) * 2
                gu_bytes += b
                w_bytes += b
            w_bytes += ex.down.trellis.numel() * 2 + (ex.down.k + ex.down.n) * 2
        npairs = B * topk + (B if t.shared is not None else 0)
        gu_bytes += B * H * 2 + npairs * I * 2
    hbm, _, peak_kind = peaks()
    roof = None
    if gu_ms:
        ach = gu_bytes / Ltot / (gu_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
                "traffic": TRAFFIC_PER_LAUNCH.get(wl), "kernel": "k_gemv<EPI_GATEUP> (gate|up GEMV)",
                "peak_kind": peak_kind, "launch_ms": round(gu_ms, 5), "bytes_per_launch": gu_bytes // Ltot}
        if wl in DECODE_ALU:
            roof["decode_alu"] = DECODE_ALU[wl]
    weight_gbs = ctx.sum_over_ranks(float(w_bytes)) / (ms * 1e-3) / 1e9
    if roof is None:
        # N > 1: the per-GPU compressed weight bytes of a step over the step time (the exchange included)
        ach = weight_gbs / world
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
                "traffic": None, "kernel": "whole step per GPU (expert weights read / step time)",
                "peak_kind": peak_kind}

    # e2e: the same step with host buffers (pinned), copies inside the timed region
    xh = x.cpu().pin_memory()
    lh = logits.cpu().pin_memory()
    oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.barrier()
    torch.cuda.synchronize()
    a0.record()
    for _ in range(steps):
        x.copy_(xh, non_blocking=True)
        logits.copy_(lh, non_blocking=True)
        graph.replay()
        oh.copy_(out, non_blocking=True)
    a1.record()
    torch.cuda.synchronize()
    ms_e2e = ctx.max_over_ranks(a0.elapsed_time(a1) / steps)
    assert torch.isfinite(oh).all(), "non-finite MoE output"
    status = L.lib().exl3_device_status(0)
    assert status == 0, f"device status {status}"
    cpu = cpu_decode_baseline(ctx.pool, ctx.cores, wl, cfg) if ctx.pool is not None else None
    line = {
        "metric": METRIC if primary else f"MoE-layer decode tok/s ({wl})", "value": round(tok_s, 2),
        "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded random trellis, +-1 signs, N(0,1))", "config": config_of(wl, cfg, world),
        "weight_gbs": round(weight_gbs, 1), "weight_gbs_frac": round(weight_gbs / world / hbm, 4),
        "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": round(B * world / (ms_e2e * 1e-3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": int(xh.numel() * 2 + lh.numel() * 4),
                "d2h_bytes_per_step": int(oh.numel() * 4)},
        "gpu_launches": (5 if world == 1 else 8 + (4 if cfg["shared_K"] else 0)) * Ltot * steps,
        "clocks": clk.summary(),
    }
    if world > 1:
        line["gpu_launches_note"] = ("per layer: route, exchange dispatch, the local experts (prepare, gate|up, "
                                     "down, combine), exchange combine and reduce, and the shared expert's four "
                                     "when the workload has one; torch fill kernels are not counted")
    del graph, graph_ev
    if world == 1 and cfg.get("batch_sweep"):
        line["batch_sweep"] = decode_batch_sweep(cfg, steps, warmup, x, logits, out, tables, kind, bias, res, line)
    return line


def decode_batch_sweep(cfg, steps, warmup, x, logits, out, tables, kind, bias, res, line):
    """The config's other decode batches (1 GPU): the first b tokens of the same step through the same layers,
    captured and timed the same way (CUDA events over `steps` replays after `warmup`)."""
    import torch
    from exl3_b200 import moe, ops
    Ltot, topk = cfg["layers"], cfg["topk"]
    sweep = {str(cfg["batch"]): {"tok_s": line["value"], "ms_per_step": line["ms_per_step"]}}
    for b in cfg["batch_sweep"]:
        def step():
            for l in range(Ltot):
                ids, w, _ = ops.route(logits[l, :b], kind, topk, bias=None if bias is None else bias[l],
                                      res=None if res is None else res[l], scale=cfg["scale"], renorm=True)
                moe.moe_forward(x[l, :b], ids, w, tables[l], cfg["act_limit"], torch.float32, out=out[l, :b])
        step()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        for _ in range(warmup):
            g.replay()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record()
        for _ in range(steps):
            g.replay()
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / steps
        sweep[str(b)] = {"tok_s": round(b / (ms * 1e-3), 2), "ms_per_step": round(ms, 5)}
        del g
    return sweep


# ------------------------------------------------------------------------------------------------ prefill

def run_prefill(ctx, args, wl, cfg, steps, warmup, primary: bool):
    """One MoE prefill layer per step (route + exl3_moe_prefill) timed with CUDA events. N > 1: expert parallelism
    (weak scaling): every rank routes its own `batch` tokens, holds E/N of the routed experts (plus the shared
    expert) and exchanges token rows with the others through ExpertParallelMoE (the peer-memory dispatch /
    combine / reduce kernels, the tcgen05 prefill kernels locally); value = all ranks' tokens / the slowest rank's step.
    roofline: tensor-bound; achieved = one rank's algorithmic flops (2 tokens topk 3 H I + shared 2 tokens 3 H I)
    / the step time (router, alignment, rotations, combine and the exchange included)."""
    import numpy as np
    import torch
    from exl3_b200 import _lib as L
    from exl3_b200 import ep, moe, ops
    world, rank, dev = ctx.world, ctx.rank, ctx.dev
    H, E, I, topk, T = cfg["H"], cfg["E"], cfg["I"], cfg["topk"], cfg["batch"]
    E_local = E // world
    e0 = rank * E_local
    gen = torch.Generator(device=dev).manual_seed(11 + rank)
    experts = []
    for e in range(e0, e0 + E_local):
        rng = np.random.default_rng(1000 + e)               # the expert's bit widths do not depend on the rank count
        Ks = [2 if rng.random() < cfg["p_k2"] else 1 for _ in range(3)]
        experts.append(moe.Expert(rand_matrix(gen, dev, H, I, Ks[0]), rand_matrix(gen, dev, H, I, Ks[1]),
                                  rand_matrix(gen, dev, I, H, Ks[2])))
    sk = cfg["shared_K"]
    shared = moe.Expert(rand_matrix(gen, dev, H, I, sk), rand_matrix(gen, dev, H, I, sk),
                        rand_matrix(gen, dev, I, H, sk))
    table = moe.ExpertTable(experts, shared)
    del experts, shared
    x = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
    logits = torch.randn(T, E, device=dev, generator=gen)
    ggen = torch.Generator(device=dev).manual_seed(7)       # router bias shared by all ranks
    bias = torch.randn(E, device=dev, generator=ggen) * 0.1
    out = torch.empty(T, H, device=dev, dtype=torch.float32)
    ws = epm = None
    if world == 1:
        ws = torch.empty(L.lib().exl3_moe_prefill_workspace_size(T, topk, E, H, I, 1), dtype=torch.uint8, device=dev)
    else:
        epm = ep.ExpertParallelMoE(E, H, topk, None, table, cfg["act_limit"], capacity=T)

    def step():
        ids, w, _ = ops.route(logits, L.ROUTE_SQRT_SOFTPLUS, topk, bias=bias, scale=cfg["scale"])
        if world == 1:
            moe.moe_prefill(x, ids, w, table, cfg["act_limit"], out=out, workspace=ws)
        else:
            epm.forward(x, ids, w, out=out)

    def timed(body):
        ctx.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            body()
        t1.record()
        torch.cuda.synchronize()
        return ctx.max_over_ranks(t0.elapsed_time(t1) / steps)

    with ClockSampler(ctx.local) as clk:
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        ms = timed(step)
    assert torch.isfinite(out).all(), "non-finite MoE output"
    assert L.lib().exl3_device_status(0) == 0

    xh, lh = x.cpu().pin_memory(), logits.cpu().pin_memory()
    oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e_step():
        x.copy_(xh, non_blocking=True)
        logits.copy_(lh, non_blocking=True)
        step()
        oh.copy_(out, non_blocking=True)

    ms_e2e = timed(e2e_step)
    assert torch.isfinite(oh).all(), "non-finite MoE output"
    cpu = cpu_prefill_baseline(ctx.pool, ctx.cores, wl, cfg) if ctx.pool is not None else None
    flops = 2.0 * T * topk * 3 * H * I + 2.0 * T * 3 * H * I
    _, tflops, peak_kind = peaks()
    ach = flops / (ms * 1e-3) / 1e12
    per_call = lambda rows: 8 if rows * topk > 8192 else 7
    launches = (per_call(T) if world == 1 else 1 + 3 + per_call(T * world) + per_call(T)) * steps
    line = {
        "metric": "MoE-layer prefill tok/s (tcgen05 grouped GEMM, tensor-pipe fraction)",
        "value": round(world * T / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded random trellis, +-1 signs, N(0,1) bf16 activations)",
        "config": {"workload": wl, "tokens_per_gpu": T, "hidden": H, "experts": E, "intermediate": I, "topk": topk,
                   "K": "1/2 (P(2)=0.62)", "shared_K": cfg["shared_K"], "router": cfg["router"],
                   "parallelism": f"ep{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (expert weights of 2.3 GB per 256 experts, 117 MB of activations "
                         "per rank and step)"},
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": tflops, "unit": "TFLOP/s",
                     "frac": round(ach / tflops, 4), "peak_kind": f"{peak_kind} bf16 burst", "traffic": None,
                     "flops_per_step_per_gpu": flops, "kernel": "whole layer (route .. combine), per rank"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(world * T / (ms_e2e * 1e-3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": int(xh.numel() * 2 + lh.numel() * 4),
                "d2h_bytes_per_step": int(oh.numel() * 4)},
        "gpu_launches": launches, "clocks": clk.summary(),
    }
    return line


# ------------------------------------------------------------------------------------------------ dense

def run_dense(ctx, args, wl, cfg, steps, warmup, primary: bool):
    """for each K, a 60-layer stack of the three EXL3 linears (5120->25600, 25600->5120,
    5120->5120; svh scaled by 1/sqrt(k) so that activations stay unit-scale) chained as a decode step, captured in
    one CUDA graph per batch size and replayed; a step = one token (per batch row) through the stack. Inputs larger
    than L2 (4.3-10.8 GB of weights per K). roofline: the stack's compressed weight bytes / step time (180 decode
    GEMVs and their activation prep per step; the GEMVs are the step) against the HBM peak. N > 1: replicas."""
    import torch
    from exl3_b200 import _lib as L
    from exl3_b200 import ops
    dev = ctx.dev
    hbm, _, peak_kind = peaks()
    shapes, layers = cfg["shapes"], cfg["layers"]
    results = {}
    clk_all = []
    for K in cfg["Ks"]:
        gen = torch.Generator(device=dev).manual_seed(60 + K + 100 * ctx.rank)
        stack = []
        wbytes = 0
        for _ in range(layers):
            for k, n in shapes:
                m = rand_matrix(gen, dev, k, n, K, 1.0 / math.sqrt(k))
                stack.append((ops.pack(m.trellis, K), m.suh, m.svh, k, n))
                wbytes += m.trellis.numel() * 2 + (k + n) * 2
                del m
        for M in cfg["batches"]:
            acts = [torch.randn((M, shapes[0][0]), device=dev, generator=gen).half()]
            for k, n in shapes * layers:
                acts.append(torch.empty((M, n), dtype=torch.half, device=dev))
            wss = {}

            def step():
                for i, (pk, suh, svh, k, n) in enumerate(stack):
                    key = (k, n)
                    if key not in wss:
                        wss[key] = torch.empty(L.lib().exl3_gemv_workspace_size(M, k, n), dtype=torch.uint8,
                                               device=dev)
                    ops.exl3_gemv(acts[i], pk, suh, svh, K, acts[i + 1], workspace=wss[key])

            step()
            torch.cuda.synchronize()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                step()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(ctx.local) as clk:
                for _ in range(warmup):
                    g.replay()
                torch.cuda.synchronize()
                ctx.barrier()
                t0.record()
                for _ in range(steps):
                    g.replay()
                t1.record()
                torch.cuda.synchronize()
            ms = ctx.max_over_ranks(t0.elapsed_time(t1) / steps)
            clk_all.append(clk.summary())
            assert torch.isfinite(acts[-1]).all(), "non-finite dense output"
            ach = wbytes / (ms * 1e-3) / 1e9
            results[f"K{K}_M{M}"] = {"tok_s": round(M * ctx.world / (ms * 1e-3), 2), "ms_per_step": round(ms, 4),
                                     "weight_gbs": round(ach, 1), "frac": round(ach / hbm, 4)}
            del g
        del stack
        torch.cuda.empty_cache()
    assert L.lib().exl3_device_status(0) == 0
    head = results["K4_M1"]
    cpu = cpu_dense_baseline(ctx.pool, ctx.cores, cfg) if ctx.pool is not None else None
    mhz = [c["sm_mhz"] for c in clk_all if c["sm_mhz"]]
    return {
        "metric": "dense EXL3 decode tok/s of a 60-layer stack (K 4, batch 1 headline; all K / batch in sweep)",
        "value": head["tok_s"], "unit": "tok/s", "n_gpus": ctx.world, "steps": steps, "warmup": warmup,
        "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded random trellis)",
        "config": config_of(wl, cfg, ctx.world),
        "roofline": {"bound": "hbm", "achieved": head["weight_gbs"], "peak": hbm, "unit": "GB/s",
                     "frac": head["frac"], "peak_kind": peak_kind, "traffic": None,
                     "kernel": "k_gemv<EPI_LINEAR> stack (K 4, batch 1): weight bytes / step time"},
        "sweep": results, "cpu_baseline": cpu,
        "gpu_launches": 2 * layers * len(shapes) * steps,
        "clocks": {"sm_mhz": statistics.median(mhz) if mhz else None,
                   "sm_max_mhz": clk_all[0]["sm_max_mhz"] if clk_all else None,
                   "reasons": sorted({r for c in clk_all for r in c["reasons"]}),
                   "samples": sum(c["samples"] for c in clk_all)},
    }


RUNNERS = {"decode": run_decode, "prefill": run_prefill, "dense": run_dense}

# DRAM bytes (read + write) per gate|up launch from the committed ncu capture
# (profiles/k_gemv_moe_qwen_next_full.md), per workload; None where no capture was made.
TRAFFIC_PER_LAUNCH: dict = {"qwen_next_decode": 31225856 + 102144}
# The decode's own roofline for the same launch, from the same capture: the kernel is bound by the integer decode of
# the trellis, not by HBM (warp instructions per 16x16 tile, issue and pipe utilisation, and the ceiling that the
# IMUL + IDP4A pair per weight sets on the half-rate pipe at this K).
DECODE_ALU: dict = {"qwen_next_decode": {
    "warp_instructions_per_tile": 54.3, "issue_active": 0.626, "alu_pipe": 0.529,
    "fma_pipe": 0.234, "smsp_active_of_elapsed": round(46355.5 / 63015.8, 3), "K": 3,
    "hbm_frac_ceiling_of_mul1_pipe": 0.53}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qwen_next_decode", choices=sorted(WORKLOADS))
    ap.add_argument("--no-extra", action="store_true", help="only the primary workload")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (small profiling captures)")
    ap.add_argument("--batch", type=int, default=0, help="tokens per GPU (default: the workload's)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    cfg = dict(WORKLOADS[args.workload])
    if args.batch:
        cfg["batch"] = args.batch
    if args.layers:
        cfg["layers"] = args.layers
    if args.impl == "reference":
        run_reference(args, cfg)
        return
    ctx = Ctx(args, want_pool=not args.no_cpu_baseline)
    ep_rel = ep_check(ctx) if ctx.world > 1 else None
    line = RUNNERS[cfg["kind"]](ctx, args, args.workload, cfg, args.steps, args.warmup, True)
    if ep_rel is not None:
        line["ep_check"] = {"max_rel_err": ep_rel, "passed": True,
                            "what": "expert-parallel output vs local moe_forward / moe_prefill on a layer every "
                                    "rank holds in full (batches 4 and 700)"}
    if args.workload == "qwen_next_decode" and not args.no_extra and not args.layers and not args.batch:
        extra = {}
        xs = min(args.steps, EXTRA_MAX_STEPS)
        for wl in EXTRAS:
            c = dict(WORKLOADS[wl])
            extra[wl] = RUNNERS[c["kind"]](ctx, args, wl, c, xs, args.warmup, False)
            import torch
            torch.cuda.empty_cache()
        line["extra"] = extra
    if ctx.rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


if __name__ == "__main__":
    main()
