"""Benchmark: int8 MoE decode tokens/s on B200 (one process per GPU).

Workload (the batched decode MoE layer): 64
concurrent sequences per GPU through one MoE FFN layer (hidden 1280, 64
routed experts of intermediate 896, top-6, + 2 fused shared experts of 896),
int8 per-row weights, routing drawn with a Zipf(1.1) expert skew.  A step is
one such layer over one batch of 64 tokens.  Weights come from a ring of
layers (each > L2) so consecutive steps stream weights from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line (rank 0).  ``value`` = tokens/s over all ranks with
inputs resident in HBM; ``e2e`` = the same through the host-buffer C-ABI call
(h2d of x/routing, d2h of y inside the timed region); ``roofline`` = the
expert kernels' algorithmic bytes per step / step time vs measured HBM peak;
``cpu_baseline`` = the reference's x86 tier restated (oracle/cpu_baseline.c)
on this host's cores over a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, INTER, NEXP, TOPK, SHARED = 1280, 896, 64, 6, 1792
# DRAM bytes (read + write) of one config-2 step's two tensor-core kernels,
# from one ncu capture of this workload (dram__bytes.sum.per_second x
# gpu__time_duration)
CFG2_TRAFFIC_BYTES = 203.4e6
CFG2_TRAFFIC_SOURCE = "ncu: MoeGateUp 136.1 MB + MoeDown 67.3 MB per step"
TOKENS = 64
L2_BYTES = 126 * 2**20


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def expert_bytes(inter=INTER, hidden=HIDDEN):
    w = 3 * inter * hidden
    s = (2 * inter + hidden) * 4
    return w + s


def step_bytes(idx_step, experts_local, tokens=TOKENS):
    """Algorithmic HBM bytes of one forward step: every routed expert hit
    (weights + scales, read once), the shared expert, x in, y out, routing."""
    hit = np.unique(idx_step)
    hit = hit[np.isin(hit, experts_local)]
    b = len(hit) * expert_bytes()
    b += expert_bytes(SHARED)
    b += tokens * HIDDEN * 4 * 2 + tokens * TOPK * 8
    return b


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.dev = dev
        self.p = None
        self.path = Path("/tmp") / f"focr_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return ws, rank, local


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(seed=100, runs=5, run_seconds=1.5):
    """Restated reference CPU tier on the host cores over a bounded sample:
    the config-2 layer (the GPU arm's first layer, seed 100) on batches of 64
    tokens with the GPU arm's inputs.  Best of `runs` timed runs (each
    `run_seconds` of batches, after one warm-up batch) at all host threads
    and at 8 threads (the reference's FOCR_THREADS default), with the
    coefficient of variation of the runs."""
    from franken_ocr_b200 import synth
    from oracle import oracle as O
    from oracle.oracle import MoeOracle

    W = synth.moe_layer(seed, shared_inter=SHARED)
    orc = MoeOracle(W)
    batches = [(synth.hidden_states(7, TOKENS, idx=i), *synth.zipf_routing(7, TOKENS, idx=i))
               for i in range(8)]

    def measure(threads):
        orc.cpu_forward(*batches[0], threads)
        rates = []
        for _ in range(runs):
            toks, i = 0, 0
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < run_seconds:
                orc.cpu_forward(*batches[i % len(batches)], threads)
                toks += TOKENS
                i += 1
            rates.append(toks / (time.perf_counter() - t0))
        r = np.array(rates)
        return {"value": float(r.max()), "cores": threads, "runs": runs,
                "cv": float(r.std() / r.mean())}

    allc = os.cpu_count() or 1
    best = measure(allc)
    eight = measure(min(8, allc))
    return {"value": best["value"], "unit": "tokens/s", "cores": allc, "kind": "port",
            "cv": best["cv"], "best_of": runs, "threads_8": eight,
            "cpu_model": cpu_model(), "tier": O.cpu_tier(),
            "sample": f"config-2 layer (seed {seed}), batches of 64 tokens, best of {runs} runs "
                      f"of {run_seconds} s at {allc} and {min(8, allc)} threads, "
                      f"{O.cpu_tier()} restatement + threaded decode_mlp_i8 driver"}


def config2_dict(ws, graph=True, R=2):
    return {"workload": "config2_moe_layer_m64_zipf_shared", "tokens_per_step": TOKENS * ws,
            "tokens_per_gpu": TOKENS, "hidden": HIDDEN, "inter": INTER, "experts": NEXP,
            "topk": TOPK, "shared_inter": SHARED,
            "parallelism": "single GPU" if ws == 1 else f"ep{ws}", "cuda_graph": graph,
            "l2": f"ring of {R} layers of {expert_bytes() * NEXP / 1e6:.0f} MB each (> L2)",
            "weights": "synth.moe_layer(100 + r), r < 2", "inputs": "hidden_states/zipf_routing(7, 64, idx=step)"}


def run_reference(args, ws, rank):
    """The reference's CPU tier (restated: oracle/cpu_baseline.c, AVX-512-VNNI
    + the threaded decode_mlp_i8 driver) on the GPU arm's workload: same
    layers (seed 100 + step % 2), same inputs, all host threads; each step is
    one batch of 64 tokens.  Rank 0 only."""
    if rank != 0:
        return
    from franken_ocr_b200 import synth
    from oracle import oracle as O
    from oracle.oracle import MoeOracle

    threads = os.cpu_count() or 1
    R = 2
    orcs = [MoeOracle(synth.moe_layer(100 + r, shared_inter=SHARED)) for r in range(R)]
    n = args.steps + args.warmup
    batches = [(synth.hidden_states(7, TOKENS, idx=i), *synth.zipf_routing(7, TOKENS, idx=i))
               for i in range(n)]
    for i in range(args.warmup):
        orcs[i % R].cpu_forward(*batches[i], threads)
    t0 = time.perf_counter()
    for i in range(args.warmup, n):
        orcs[i % R].cpu_forward(*batches[i], threads)
    dt = time.perf_counter() - t0
    v = args.steps * TOKENS / dt
    print(json.dumps({
        "impl": "reference", "metric": "int8 MoE decode tokens/s (config 2: M=64 batched decode layer)",
        "value": v, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 (i32 accumulate, f32 dequant)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) hidden, Zipf(1.1) routing)",
        "config": config2_dict(1),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"{args.steps} steps x 64 tokens, {O.cpu_tier()} restatement, "
                                   f"{threads} threads"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_ours(args, ws, rank, local):
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        return run_ep(args, ws, rank, local)
    hbm_peak, peak_kind = peaks()
    if args.workload == "config1":
        shape = tuple(int(v) for v in args.shape.split("x")) if args.shape else None
        int8_peak, rows = igemm_sweep(dev, hbm_peak, peak_kind, reps=max(1, args.steps), shape=shape)
        tot_us = sum(r["us"] for r in rows)
        print(json.dumps({
            "metric": "int8 GEMM sweep (config 1): sum of per-shape times", "value": tot_us,
            "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": 2,
            "ms_per_step": tot_us / 1e3, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 (i32 accumulate)", "data": "synthetic",
            "config": {"workload": "config1_igemm_sweep", "out": "+= int32"},
            "int8_peak_tops_own_kernel": int8_peak, "hbm_peak": hbm_peak, "peak_kind": peak_kind,
            "shapes": rows}), flush=True)
        return
    if args.workload == "config0":
        m1 = m1_decode(dev, hbm_peak, peak_kind, steps=args.steps)
        print(json.dumps({
            "metric": "int8 MoE decode layer-tokens/s (config 0: M=1 single-token layer)",
            "value": m1["layer_tokens_per_s"], "unit": "layer-tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": 3 * 8, "ms_per_step": m1["us_per_token_layer"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 (i32 accumulate, f32 dequant)", "data": "synthetic",
            "config": {"workload": m1["workload"], "l2": m1["l2"], "cuda_graph": m1["cuda_graph"]},
            "roofline": m1["roofline"], "gpu_launches": args.steps}), flush=True)
        return
    if args.workload == "config3":
        return config3(args, dev)
    if args.workload == "config4":
        c4 = config4_measure(dev, hbm_peak, peak_kind, reps=max(3, args.steps))
        print(json.dumps({
            "metric": "int4 MoE decode tokens/s (config 4: M=256 int4 g32 layer)",
            "value": c4["moe_m256"]["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": 3, "ms_per_step": c4["moe_m256"]["us_per_step"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 weights x int8 activations (i32 per group, f32 across groups)",
            "data": "synthetic", "config": {"workload": c4["workload"]},
            "roofline": c4["moe_m256"]["roofline"], "config4": c4}), flush=True)
        return
    if args.workload == "config3_batch":
        return config3_batch(args, dev)
    # ring of layers so that consecutive steps stream from HBM
    R = 2
    layers = [MoeLayer(synth.moe_layer(100 + r, shared_inter=SHARED), max_tokens=TOKENS)
              for r in range(R)]
    n = args.steps + args.warmup
    xs = [synth.hidden_states(7, TOKENS, idx=i) for i in range(n)]
    rts = [synth.zipf_routing(7, TOKENS, idx=i) for i in range(n)]
    xd = [torch.from_numpy(x).to(dev) for x in xs]
    idd = [torch.from_numpy(r[0]).to(dev) for r in rts]
    wd = [torch.from_numpy(r[1]).to(dev) for r in rts]
    y = torch.empty((TOKENS, HIDDEN), dtype=torch.float32, device=dev)
    experts_local = np.arange(NEXP)

    def step(i):
        layers[i % R].forward(xd[i], idd[i], wd[i], y)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    graph = capture(step, range(args.warmup, n))
    torch.cuda.synchronize()
    e0.record(st)
    if graph is not None:
        graph.replay()
    else:
        for i in range(args.warmup, n):
            step(i)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    ms_step = ms / args.steps
    value = args.steps * TOKENS * ws / (ms / 1e3)
    bytes_per_step = float(np.mean([step_bytes(rts[i][0], experts_local) for i in range(args.warmup, n)]))
    achieved = bytes_per_step / (ms_step / 1e3) / 1e9

    # e2e: same steps through the host-buffer C-ABI call (pinned host memory)
    xh = [torch.from_numpy(x).pin_memory().numpy() for x in xs]
    ih = [torch.from_numpy(r[0]).pin_memory().numpy() for r in rts]
    wh = [torch.from_numpy(r[1]).pin_memory().numpy() for r in rts]
    yh = torch.empty((TOKENS, HIDDEN), dtype=torch.float32).pin_memory().numpy()
    for i in range(args.warmup):
        layers[i % R].forward(xh[i], ih[i], wh[i], yh)
    ds = torch.cuda.default_stream()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(ds)
    for i in range(args.warmup, n):
        layers[i % R].forward(xh[i], ih[i], wh[i], yh)
    e3.record(ds)
    torch.cuda.synchronize()
    e2e_ms = e2.elapsed_time(e3)
    h2d = TOKENS * HIDDEN * 4 + TOKENS * TOPK * 8
    d2h = TOKENS * HIDDEN * 4

    m1 = None if args.no_m1 else m1_decode(dev, hbm_peak, peak_kind)
    cpu = cpu_baseline() if rank == 0 and not args.no_cpu else None
    launches_per_step = 8
    line = {
        "metric": "int8 MoE decode tokens/s (config 2: M=64 batched decode layer)",
        "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (i32 accumulate, f32 dequant)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) hidden, Zipf(1.1) routing)",
        "config": config2_dict(ws, graph is not None, R),
        "roofline": {"bound": "hbm", "kernel": "moe_forward step (all expert kernels)",
                     "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_kind": peak_kind,
                     "traffic": CFG2_TRAFFIC_BYTES, "traffic_source": CFG2_TRAFFIC_SOURCE,
                     "algorithmic_bytes_per_step": bytes_per_step},
        "e2e": {"value": args.steps * TOKENS * ws / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    if m1:
        line["m1_decode"] = m1
    if not args.no_extras:
        # the other configurations, measured in the same run (driver-visible)
        def extra(key, fn):
            try:
                line[key] = fn()
            except Exception as exc:  # pragma: no cover - reported, never fatal
                line[key] = {"error": f"{type(exc).__name__}: {exc}"}

        def c1():
            own, rows = igemm_sweep(dev, hbm_peak, peak_kind, reps=5)
            lib_peak = int8_library_peak(dev)
            return {"workload": "config1_igemm_sweep (out += int32)", "shapes": rows,
                    "int8_peak_tops_own_kernel": own, "int8_peak_tops_torch_int_mm": lib_peak,
                    "note": "frac = floor / time, floor = max(bytes / HBM peak, ops / own-kernel peak)"}

        extra("config1", c1)
        extra("config3", lambda: config3_line(args, dev, steps=2))
        extra("config4", lambda: config4_measure(dev, hbm_peak, peak_kind))
    if rank == 0:
        print(json.dumps(line), flush=True)


def m1_decode(dev, hbm_peak, peak_kind, steps=200):
    """Config 0 beside the headline: one token through one MoE layer
    (64 experts, top-6 renormalised, no shared expert) with focr_moe_decode,
    i.e. the fused single-token kernel.  A ring of 8 layers (1.8 GB) keeps
    the weights streaming from HBM; timed as one CUDA graph of `steps`
    decodes.  Algorithmic bytes per token-layer: 6 routed experts (weights +
    scales) + router + x/y."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer

    R = 8
    layers = [MoeLayer(synth.moe_layer(1000 + r), max_tokens=1) for r in range(R)]
    xs = [torch.from_numpy(synth.hidden_states(50 + r, 1)).to(dev) for r in range(R)]
    ys = [torch.empty((1, HIDDEN), device=dev) for _ in range(R)]
    ids = [torch.empty((1, TOPK), dtype=torch.int32, device=dev) for _ in range(R)]
    ws_ = [torch.empty((1, TOPK), device=dev) for _ in range(R)]

    def step(i):
        r = i % R
        layers[r].decode(xs[r], ys[r], ids[r], ws_[r])

    for i in range(3 * R):
        step(i)
    torch.cuda.synchronize()
    graph = capture(step, range(steps))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = torch.cuda.current_stream()
    e0.record(st)
    if graph is not None:
        graph.replay()
    else:
        for i in range(steps):
            step(i)
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    bytes_tok = 6 * expert_bytes() + NEXP * HIDDEN * 4 + 2 * HIDDEN * 4
    achieved = bytes_tok / (us / 1e6) / 1e9
    for L in layers:
        L.close()
    return {"workload": "config0_moe_layer_m1 (fused single-token kernel, moe_m1_fused_kernel)",
            "us_per_token_layer": us, "layer_tokens_per_s": 1e6 / us,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": bytes_tok},
            "cuda_graph": graph is not None, "l2": f"ring of {R} layers x 220 MB (> L2)"}


def igemm_sweep(dev, hbm_peak, peak_kind, reps=5, shape=None):
    """Config 1: the raw int8 x int8 -> int32 GEMM sweep through
    focr_igemm_s8s8 on device tensors (out += A.B^T), each shape timed as one
    CUDA graph of `reps` calls.  Each shape's floor is
    max(bytes / HBM peak, ops / int8 peak); the int8 peak is the one this
    build's own tcgen05 kernel reaches on a compute-bound shape (8192 x 8192 x
    16384) in the same run.  Inputs: a, b uniform in [-127, 127]."""
    import torch

    from franken_ocr_b200 import simd

    def timed(m, n, k):
        g = torch.Generator(device=dev).manual_seed(m * 31 + n)
        a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g)
        o = torch.zeros((m, n), dtype=torch.int32, device=dev)
        for _ in range(2):
            simd.igemm_s8s8(a, b, m, k, n, o)
        torch.cuda.synchronize()
        # one CUDA graph of `reps` calls: the host-side call cost stays out
        graph = capture(lambda i: simd.igemm_s8s8(a, b, m, k, n, o), range(reps))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if graph is not None:
            graph.replay()
        else:
            for _ in range(reps):
                simd.igemm_s8s8(a, b, m, k, n, o)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    if shape is None:
        us_peak = timed(8192, 8192, 16384)
        int8_peak = 2 * 8192 * 8192 * 16384 / us_peak / 1e6   # TOPS
        shapes = [(m, n, k) for (n, k) in [(1792, 1280), (1280, 896), (129280, 1280)]
                  for m in (1, 8, 64, 512, 4096)]
    else:   # one shape (a small case for a profiler capture); no peak shape
        int8_peak = None
        shapes = [shape]
    rows = []
    for (m, n, k) in shapes:
        us = timed(m, n, k)
        ops, byt = 2 * m * n * k, m * k + n * k + 8 * m * n
        floor_us = max(byt / hbm_peak / 1e3, ops / int8_peak / 1e6 if int8_peak else 0.0)
        rows.append({"m": m, "n": n, "k": k, "us": round(us, 2), "tops": ops / us / 1e6,
                     "gbs": byt / us / 1e3, "floor_us": floor_us, "frac": floor_us / us})
    return int8_peak, rows


def capture(step, idxs):
    """One CUDA graph holding the given steps (their launches, and NCCL
    collectives for N > 1), so host-side launch overhead leaves the timed
    region; None if capture is not possible here."""
    import torch

    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in idxs:
                step(i)
        torch.cuda.synchronize()
        g.replay()            # graph warm-up (same steps; untimed)
        torch.cuda.synchronize()
        return g
    except Exception as exc:  # pragma: no cover - reported in the JSON line
        print(f"bench: CUDA graph capture failed ({exc}); timing eager launches", file=sys.stderr)
        return None


def run_ep(args, ws, rank, local):
    """N > 1: expert parallel, 64 tokens per GPU (weak scaling), each GPU
    owning 64/N routed experts and a replica of the router and the shared
    expert.  The library's data plane (focr_ep_*): routed int8 rows written
    into the owners' staging buffers over NVLink, partials written back by
    the owners' down GEMM epilogue, slot-ordered combine at the source; NCCL
    (focr_comm) bootstraps the peer mappings."""
    import torch
    import torch.distributed as dist

    from franken_ocr_b200 import synth
    from franken_ocr_b200.ep import Comm, EpMoe, nccl_unique_id
    from franken_ocr_b200.moe import MoeLayer

    dev = torch.device("cuda", local)
    hbm_peak, peak_kind = peaks()
    e_local = NEXP // ws
    R = 2
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = Comm(obj[0], rank, ws)
    layers = []
    for r in range(R):
        L = EpMoe(synth.moe_layer(100 + r, shared_inter=SHARED, expert_begin=rank * e_local,
                                  expert_count=e_local), rank, ws, TOKENS)
        L.connect_comm(comm)
        layers.append(L)
    n = args.steps + args.warmup
    seed = 7 + 1000 * rank
    xs = [synth.hidden_states(seed, TOKENS, idx=i) for i in range(n)]
    rts = [synth.zipf_routing(seed, TOKENS, idx=i) for i in range(n)]
    xd = [torch.from_numpy(x).to(dev) for x in xs]
    idd = [torch.from_numpy(r[0]).to(dev) for r in rts]
    wd = [torch.from_numpy(r[1]).to(dev) for r in rts]

    def step(i):
        return layers[i % R].forward(xd[i], idd[i], wd[i])

    # parity: the first step's output equals the single-GPU layer's, bit for bit
    full = MoeLayer(synth.moe_layer(100, shared_inter=SHARED), max_tokens=TOKENS)
    y0 = step(0).cpu().numpy()
    want0 = full.forward(xs[0], *rts[0])
    full.close()
    parity = bool(np.array_equal(y0.view(np.uint32), want0.view(np.uint32)))
    flag = torch.tensor([int(parity)], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    parity = bool(flag.item())
    for i in range(1, args.warmup):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    dist.barrier()
    graph = capture(step, range(args.warmup, n))
    torch.cuda.synchronize()
    dist.barrier()
    e0.record(st)
    if graph is not None:
        graph.replay()
    else:
        for i in range(args.warmup, n):
            step(i)
    e1.record(st)
    torch.cuda.synchronize()
    dist.barrier()
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    clk = clocks.stop()

    # e2e: host (pinned) inputs copied in and y copied out inside the timed region
    xh = [torch.from_numpy(x).pin_memory() for x in xs]
    ih = [torch.from_numpy(r[0]).pin_memory() for r in rts]
    wh = [torch.from_numpy(r[1]).pin_memory() for r in rts]
    yh = torch.empty((TOKENS, HIDDEN), dtype=torch.float32).pin_memory()

    def e2e_step(i):
        y = layers[i % R].forward(xh[i].to(dev, non_blocking=True), ih[i].to(dev, non_blocking=True),
                                  wh[i].to(dev, non_blocking=True))
        yh.copy_(y, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    dist.barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(st)
    for i in range(args.warmup, n):
        e2e_step(i)
    e3.record(st)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e2.elapsed_time(e3)], device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    # this rank's experts are hit by every rank's tokens: regenerate all routings
    local_experts = np.arange(rank * e_local, (rank + 1) * e_local)
    all_rts = [[synth.zipf_routing(7 + 1000 * q, TOKENS, idx=i)[0] for q in range(ws)]
               for i in range(args.warmup, n)]
    my_bytes = float(np.mean([step_bytes(np.concatenate([a.ravel() for a in ri]), local_experts)
                              for ri in all_rts]))
    ms_step = ms / args.steps
    achieved = my_bytes / (ms_step / 1e3) / 1e9
    line = {
        "metric": "int8 MoE decode tokens/s (config 2: M=64 batched decode layer)",
        "value": args.steps * TOKENS * ws / (ms / 1e3), "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 (i32 accumulate, f32 dequant)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) hidden, Zipf(1.1) routing)",
        "config": {**config2_dict(ws, graph is not None, R),
                   "inputs": "hidden_states/zipf_routing(7 + 1000 * rank, 64, idx=step)",
                   "l2": f"ring of {R} layers (local experts {e_local}); weights streamed from HBM"},
        "roofline": {"bound": "hbm", "kernel": "EP forward step (rank 0's own-token + own-expert bytes)",
                     "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_step": my_bytes},
        "e2e": {"value": args.steps * TOKENS * ws / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": TOKENS * HIDDEN * 4 + TOKENS * TOPK * 8,
                "d2h_bytes_per_step": TOKENS * HIDDEN * 4},
        "gpu_launches": 9 * args.steps,
        "parity": "rank outputs bit-identical to the single-GPU layer" if parity else "MISMATCH",
        "ep_status": max(L.status() for L in layers),
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    for L in layers:
        L.close()
    comm.close()


def timed_graph(step, n, warm=3):
    """us per call of step(i) for i < n, replayed from one CUDA graph."""
    import torch

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    g = capture(step, range(n))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if g is not None:
        g.replay()
    else:
        for i in range(n):
            step(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / n


def config4_measure(dev, hbm_peak, peak_kind, reps=20):
    """Config 4: int4 g32 experts with config 0's MoE shapes (64 experts,
    top-6, no shared expert) at M = 1 and M = 256 (route + experts, decode
    semantics), and the int4 g32 lm-head shard [16160, 1280] with its top-1
    at M = 1 and M = 256.  Rings of layers (> L2) keep the weights streaming
    from HBM; each case is one CUDA graph of `reps` calls.  Bytes are the
    algorithmic int4 weight + scale bytes a call must read."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.lmhead import LmHeadShard
    from franken_ocr_b200.moe import MoeLayer
    from franken_ocr_b200.quant import pack_int4_f32

    G = 32
    per_expert = 3 * INTER * HIDDEN // 2 + (2 * INTER * HIDDEN + HIDDEN * INTER) // G * 4
    out = {"workload": "config4_int4_g32", "group": G}
    R = 8
    layers = [MoeLayer(synth.moe_layer(4500 + r, group=G), max_tokens=256) for r in range(R)]
    for m in (1, 256):
        xs = [torch.from_numpy(synth.hidden_states(4600 + r, m)).to(dev) for r in range(R)]
        ys = [torch.empty((m, HIDDEN), device=dev) for _ in range(R)]
        ii = [torch.empty((m, TOPK), dtype=torch.int32, device=dev) for _ in range(R)]
        ww = [torch.empty((m, TOPK), device=dev) for _ in range(R)]
        us = timed_graph(lambda i: layers[i % R].decode(xs[i % R], ys[i % R], ii[i % R], ww[i % R]),
                         reps)
        hit = np.mean([len(np.unique(ii[r].cpu().numpy())) for r in range(R)])
        byt = hit * per_expert + NEXP * HIDDEN * 4
        out[f"moe_m{m}"] = {"us_per_step": us, "tokens_per_s": m / (us / 1e6),
                            "experts_hit": float(hit),
                            "roofline": {"bound": "hbm", "achieved": byt / us / 1e3, "peak": hbm_peak,
                                         "unit": "GB/s", "frac": byt / us / 1e3 / hbm_peak,
                                         "peak_kind": peak_kind, "algorithmic_bytes": byt}}
    for L in layers:
        L.close()
    rows = 16160
    heads = []
    for r in range(4):   # 4 shards (52 MB) > L2
        packed, sc = pack_int4_f32(synth.normal(4700, "lm_head", r, (rows, HIDDEN), 0.02), G)
        heads.append(LmHeadShard(packed, sc, row_begin=r * rows, max_tokens=256, group=G))
    hb = rows * HIDDEN // 2 + rows * (HIDDEN // G) * 4
    for m in (1, 256):
        x = torch.from_numpy(synth.hidden_states(4800, m)).to(dev)
        us = timed_graph(lambda i: heads[i % 4].top1(x), reps)
        ops = 2 * m * rows * HIDDEN
        out[f"lmhead_shard_m{m}"] = {
            "us": us, "rows": rows, "tokens_per_s": m / (us / 1e6),
            "roofline": {"bound": "hbm", "achieved": hb / us / 1e3, "peak": hbm_peak, "unit": "GB/s",
                         "frac": hb / us / 1e3 / hbm_peak, "peak_kind": peak_kind,
                         "algorithmic_bytes": hb, "int_tops": ops / us / 1e6}}
    for h in heads:
        h.close()
    out["parity"] = "tests/test_gpu_config4.py: MoE and lm-head shard bit-identical to the oracle at M=1, 256"
    return out


def int8_library_peak(dev):
    """An int8 tensor-core throughput that is not this build's kernel: torch's
    int8 matmul (cuBLASLt, i8 x i8 -> i32) on 8192 x 8192 x 16384, best of 5;
    None when unavailable."""
    import torch

    try:
        a = torch.randint(-127, 128, (8192, 16384), dtype=torch.int8, device=dev)
        b = torch.randint(-127, 128, (16384, 8192), dtype=torch.int8, device=dev)
        for _ in range(2):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = None
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1)
            best = t if best is None else min(best, t)
        return 2 * 8192 * 8192 * 16384 / (best / 1e3) / 1e12
    except Exception as exc:  # pragma: no cover
        print(f"bench: torch._int_mm unavailable ({exc})", file=sys.stderr)
        return None


def cpu_baseline_config3(W, seed, prefill=32, seconds=10.0, max_steps=200):
    """The reference's decode loop restated on the host cores: projections,
    dense MLP, MoE experts (decode_mlp_i8's task split) and lm-head on the
    restated AVX-512-VNNI tier with all threads, RMSNorm/RoPE/attention as
    the oracle (oracle.DecoderOracle(threads=N), bit-identical to the scalar
    oracle).  Bounded sample: a 32-token prefill, then `steps` greedy decode
    steps timed; the attention span (32 + steps keys instead of 1024+) is the
    one difference from the GPU workload."""
    from franken_ocr_b200 import synth
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    steps = 0
    D = O.DecoderOracle(W, threads=threads)
    h = D.prefill(synth.prompt_embeds(seed, prefill))
    tok = O.argmax_row(D.lm_head(h[-1]))
    t0 = time.perf_counter()
    while steps < max_steps and time.perf_counter() - t0 < seconds:
        h = D.decode_step(W.embed[tok], prefill + steps)
        tok = O.argmax_row(D.lm_head(h[-1]))
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{steps} greedy decode steps after a {prefill}-token prefill, "
                      f"{O.cpu_tier()} restatement of the int8 decode loop, {threads} threads, "
                      f"{dt:.1f} s"}


def config3_roofline(W, prefill, n_tokens, d_ms):
    """(roofline dict, launches of our kernels in the decode loop) for config 3."""
    # algorithmic bytes of one decode token: every int8 weight byte it reads
    # (+ f32 scales): 6 routed experts + the shared expert per MoE layer, the
    # dense layer-0 MLP, q/k/v/o per layer, the lm-head; reference+ring K/V
    # (f32) read by attention
    hbm_peak, peak_kind = peaks()
    tok_bytes = 0
    for L in W.layers:
        for k in ("q", "k", "v", "o"):
            tok_bytes += L.proj[k + "_w"].nbytes + L.proj[k + "_s"].nbytes
        if L.dense is not None:
            tok_bytes += sum(a.nbytes for a in L.dense.values())
        else:
            per_expert = sum(L.moe.arrays[k].nbytes for k in ("gate_w", "up_w", "down_w",
                                                              "gate_s", "up_s", "down_s"))
            tok_bytes += L.moe.topk * per_expert // L.moe.expert_count
            tok_bytes += sum(L.moe.arrays[k].nbytes for k in L.moe.arrays if k.startswith("sh_"))
            tok_bytes += L.moe.router.nbytes
    tok_bytes += W.lm_w.nbytes + W.lm_s.nbytes
    kv = 2 * len(W.layers) * W.heads * 128 * 4 * (prefill + min(n_tokens, 128) / 2)
    tok_bytes += kv
    achieved = tok_bytes / (d_ms / (n_tokens - 1) / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
            "frac": achieved / hbm_peak, "traffic": None,
            "note": f"{tok_bytes / 1e6:.0f} MB of weights + K/V per decode token; peak "
                    f"{peak_kind}; the step is launch/latency bound, not bandwidth bound"}
    # our kernels per decode token: per layer (add +) RMSNorm + q|k|v GEMV,
    # RoPE + ring write, attention scores + fold, o GEMV, add+RMSNorm, then
    # the fused MoE kernel or the dense MLP (gate|up GEMV, SwiGLU, down);
    # plus prologue, final add+RMSNorm, lm-head GEMV and the two-stage argmax
    per_tok = sum(7 if L.moe is not None else 9 for L in W.layers) + 5
    launches = per_tok * (n_tokens - 1)
    return roof, launches


def config3_batch(args, dev, streams=16, batch=8, prefill=256, n_tokens=64, seed=3):
    """Continuous batching on the config-3 decoder: `streams` prompts of
    `prefill` tokens, `batch` active at a time, `n_tokens` greedy tokens each
    (BatchScheduler + DecoderBatchStep + BatchedDecoderI8).  Timed on the
    device from the first batched step to the last; the metric is aggregate
    decode tokens/s."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.batch import BatchedDecoderI8, BatchScheduler, DecoderBatchStep, PageStream

    W = synth.decoder_model(seed)
    B = BatchedDecoderI8(W, n_streams=streams, max_prefill=prefill)
    embeds = [torch.from_numpy(synth.prompt_embeds(seed + 100 + i, prefill)).to(dev)
              for i in range(streams)]

    def run():
        ss = [PageStream(i, prefill, [], B.prefill_stream(i, embeds[i])) for i in range(streams)]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        toks = BatchScheduler(batch, n_tokens).run(ss, DecoderBatchStep(B, eos_token_id=-1))
        e1.record()
        torch.cuda.synchronize()
        return toks, e0.elapsed_time(e1)

    for _ in range(max(1, args.warmup)):
        toks0, _ = run()
    ms = []
    for _ in range(args.steps):
        toks, t = run()
        assert toks == toks0, "tokens changed between runs"
        ms.append(t)
    t = float(np.median(ms))
    total = streams * n_tokens
    print(json.dumps({
        "metric": "int8 decoder continuous-batch decode tokens/s (config 3 decoder)",
        "value": total / (t / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(1, args.warmup), "ms_per_step": t, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (i32 accumulate, f32 dequant)",
        "data": "synthetic (random-init weights, N(0,1) prompt embeddings)",
        "config": {"workload": "config3_continuous_batch", "streams": streams, "batch": batch,
                   "prefill_tokens": prefill, "decode_tokens": n_tokens,
                   "decode_loop": "eager host loop per batched step"}}), flush=True)
    B.close()


def config3(args, dev, prefill=1024, n_tokens=256, seed=3):
    print(json.dumps(config3_line(args, dev, prefill, n_tokens, seed)), flush=True)


def config3_line(args, dev, prefill=1024, n_tokens=256, seed=3, steps=None):
    """Config 3: the synthetic 12-layer int8 decoder; one step = a
    1024-token prefill then a 256-token greedy decode (batch 1), the decode
    loop replayed from one captured CUDA graph per token.  Timed on the
    device with CUDA events (decode time = the prefill+decode span minus a
    separately timed prefill); the metric is decode tokens/s (256 / decode
    time), prefill tokens/s beside it."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.decoder import DecoderI8

    W = synth.decoder_model(seed)
    D = DecoderI8(W, max_prefill=prefill)
    e = torch.from_numpy(synth.prompt_embeds(seed, prefill)).to(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]

    def run():
        ev[0].record()
        D.prefill(e)
        ev[1].record()
        timer = []
        toks = D.generate_graph(e, n_tokens, timer=timer)  # prefill again + greedy decode
        torch.cuda.synchronize()
        p_ms = ev[0].elapsed_time(ev[1])
        # decode: the replayed graph steps, timed on the device around the
        # replay loop, scaled to the n_tokens - 1 decode steps of the call
        t0, t1, k = timer[0]
        return [int(t) for t in toks], p_ms, t0.elapsed_time(t1) / k * (n_tokens - 1)

    for _ in range(max(3, args.warmup)):
        toks0, _, _ = run()
    golden = json.loads((ROOT / "tests" / "golden" / "decoder_config3_greedy256.json").read_text())
    assert (golden["seed"], golden["prefill_tokens"], golden["n_tokens"]) == (seed, prefill, n_tokens)
    assert toks0 == golden["tokens"], "greedy tokens differ from the CPU oracle's"
    clocks = Clocks(dev.index or 0)
    clocks.start()
    pre, dec = [], []
    for _ in range(steps or args.steps):
        toks, p_ms, d_ms = run()
        assert toks == toks0, "greedy tokens changed between runs"
        pre.append(p_ms)
        dec.append(d_ms)
    clk = clocks.stop()
    # e2e: the public call from pinned host embeddings to host token ids
    e_host = torch.from_numpy(synth.prompt_embeds(seed, prefill)).pin_memory()
    e2 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    e2[0].record()
    toks_e2e = D.generate_graph(e_host.to(dev, non_blocking=True), n_tokens)
    e2[1].record()
    torch.cuda.synchronize()
    assert [int(t) for t in toks_e2e] == toks0
    e2e_ms = e2[0].elapsed_time(e2[1])
    d_ms, p_ms = float(np.median(dec)), float(np.median(pre))
    cpu = None if args.no_cpu else cpu_baseline_config3(W, seed)
    roof, launches = config3_roofline(W, prefill, n_tokens, d_ms)
    D.close()
    return {
        "metric": "int8 decoder greedy decode tokens/s (config 3: 12 layers, batch 1)",
        "value": (n_tokens - 1) / (d_ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": steps or args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": p_ms + d_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (i32 accumulate, f32 dequant)",
        "data": "synthetic (random-init weights, N(0,1) prompt embeddings)",
        "config": {"workload": "config3_decoder_prefill1024_greedy256", "layers": 12,
                   "prefill_tokens": prefill, "decode_tokens": n_tokens,
                   "decode_loop": "one CUDA graph per token",
                   "l2": "no flush; each token streams > 300 MB of weights (> 126 MB L2)"},
        "prefill_ms": p_ms, "prefill_tokens_per_s": prefill / (p_ms / 1e3),
        "decode_ms_per_token": d_ms / (n_tokens - 1),
        "decode_timing": "CUDA events around the graph replays of the decode step (one step per "
                         "token after the first), per-step time x 255 steps",
        "e2e": {"value": n_tokens / (e2e_ms / 1e3), "unit": "tokens/s (prefill included)",
                "h2d_bytes_per_step": prefill * W.hidden * 4, "d2h_bytes_per_step": n_tokens * 4},
        "roofline": roof, "gpu_launches": launches,
        "cpu_baseline": cpu, "clocks": clk, "tokens_head": toks0[:16],
        "parity": "all 256 greedy tokens equal the CPU oracle's (tests/golden)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-m1", action="store_true", help="skip the config-0 single-token line")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the config-1/3/4 measurements added to the default line")
    ap.add_argument("--workload", default="config2", choices=["config2", "config0", "config1", "config3", "config3_batch", "config4"],
                    help="config0: only the single-token layer; config1: the raw igemm sweep; "
                         "config3: the 12-layer decoder")
    ap.add_argument("--shape", default=None,
                    help="config1 only: time one MxNxK shape (e.g. 4096x4096x4096) instead of the sweep")
    args = ap.parse_args()
    ws, rank, local = dist_init()
    if args.impl == "reference":
        run_reference(args, ws, rank)
    else:
        run_ours(args, ws, rank, local)
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
