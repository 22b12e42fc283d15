#!/usr/bin/env python3
"""Benchmark of the quantized-matvec / MoE path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: one MoE FFN layer at decode batch 1 --
hidden 2048, 256 experts, top-8, expert intermediate 512, Q4_K gate/up,
Q6_K down, router logits fp32[256] ~ N(0,1), x fp32[2048] ~ N(0,1).
A step is one token through the layer: route -> 8 x (gate, up, silu*up,
down) -> routing-weighted sum, all on the GPU through libqw6cuda's C ABI.

Inputs larger than L2: 16 copies of the layer (16 x 522 MB of expert
weights) are resident and step s uses layer s % 16 with its own logits and
x, so an expert's weights are re-touched only after >= 256 MB of other
traffic (L2 is 126 MB).  Steps run as a CUDA graph replayed back to back.

Printed JSON line (rank 0): metric "MoE-layer tokens/s", value = whole-job
tokens/s (N replicas at N GPUs, weak scaling), the dominant kernel's HBM
roofline, an end-to-end number through the host-buffer C entry point
(qw6cu_moe_decode_hostio), the CPU baseline (qw6's own CPU code), clocks
sampled during the timed region, and per-format matvec HBM throughput.

--impl reference times qw6's own CPU implementation (oracle/_ref, built from
the reference sources) of the same layer on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, INTER, NE, TOPK = 2048, 512, 256, 8
N_LAYERS = 16
GRAPH_STEPS = 256
FALLBACK_HBM_GBS = 6650.0
METRIC = "MoE-layer tokens/s"
Q4K_BYTES_EXPERT = 512 * 8 * 144          # gate or up: 512 rows x 8 super-blocks
Q6K_BYTES_EXPERT = 2048 * 2 * 210         # down: 2048 rows x 2 super-blocks
WEIGHT_BYTES_TOKEN = TOPK * (2 * Q4K_BYTES_EXPERT + Q6K_BYTES_EXPERT)  # 16,318,464


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    return int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")), ws


# ---------------------------------------------------------------- clocks --

class ClockSampler:
    """nvidia-smi sampling during the timed region (clocks + throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.15)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            r = [c.strip() for c in r]
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ CPU legs ----

def cpu_reference_rate(gate, up, down, logits, x, budget_s: float, threads: int):
    """qw6's own CPU code (oracle/_ref): tokens/s of the MoE layer over a
    bounded sample.  Units of work are (token, selected expert) pairs run on
    `threads` host threads (ctypes drops the GIL inside qw6's C)."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle.oracle import Reference
    ref = Reference()
    ntok = logits.shape[0]
    routes = [ref.moe_route(logits[t], TOPK) for t in range(ntok)]

    def unit(u):
        t, k = divmod(u, TOPK)
        t %= ntok
        e = int(routes[t][0][k])
        g = ref.matvec(4, gate[e], x[t], INTER, HIDDEN)
        uu = ref.matvec(4, up[e], x[t], INTER, HIDDEN)
        mid = np.array([ref.silu(float(v)) for v in g], np.float32) * uu
        return np.float32(routes[t][1][k]) * ref.matvec(7, down[e], mid.astype(np.float32), HIDDEN, INTER)

    done = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        while time.perf_counter() - t0 < budget_s:
            list(ex.map(unit, range(done, done + threads)))
            done += threads
    dt = time.perf_counter() - t0
    return done / TOPK / dt, done, dt


# ------------------------------------------------------------- our arm ----

def build_layers(torch, ctx, L, n_layers):
    """Config-1 expert packs (seeded numpy generator), packed on the GPU,
    replicated into n_layers resident copies."""
    from qw6_b200 import synth as S
    gate, up, down, _, _ = S.config1()
    packs = []
    for q, m, r, c in ((S.Q4_K, gate, INTER, HIDDEN), (S.Q4_K, up, INTER, HIDDEN), (S.Q6_K, down, HIDDEN, INTER)):
        pb = ctx.packed_bytes(q, r, c)
        raw = torch.from_numpy(m.reshape(-1)).cuda()
        pk = torch.empty(pb * NE, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ctx.pack(q, raw.data_ptr(), pk.data_ptr(), r, c, NE, m[0].nbytes, pb)
        ctx.synchronize()
        del raw
        copies = [pk] + [pk.clone() for _ in range(n_layers - 1)]
        packs.append((q, pb, copies))
    layers = []
    for li in range(n_layers):
        layers.append(tuple(L.ExpertPack(q, copies[li].data_ptr(), pb) for q, pb, copies in packs))
    return (gate, up, down), packs, layers


def run_ours(args, rank, local_rank, world):
    import torch

    from qw6_b200 import lib as L

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    stream = torch.cuda.Stream()
    ctx = L.Context(local_rank)
    ctx.set_stream(stream.cuda_stream)
    raw, packs, layers = build_layers(torch, ctx, L, args.layers)
    nl = args.layers

    K, W = args.steps, args.warmup
    nslots = GRAPH_STEPS
    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    logits = torch.randn((nslots, NE), generator=gen, device="cuda", dtype=torch.float32)
    xs = torch.randn((nslots, HIDDEN), generator=gen, device="cuda", dtype=torch.float32)
    outs = torch.empty((nslots, HIDDEN), device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()

    def step(s):
        g, u, d = layers[s % nl]
        j = s % nslots
        ctx.moe_decode(g, u, d, logits[j].data_ptr(), xs[j].data_ptr(), outs[j].data_ptr(), 1, HIDDEN, INTER, NE,
                       TOPK)

    # warm-up (eager): allocates the workspace, sets kernel attributes
    with torch.cuda.stream(stream):
        for s in range(max(W, 1)):
            step(s)
    ctx.synchronize()

    def capture(nsteps, profile):
        g = torch.cuda.CUDAGraph()
        if profile:
            ctx.profile_begin(4 * nsteps + 8)
        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
            for s in range(nsteps):
                step(s)
        return g

    full = capture(GRAPH_STEPS, False)
    tail_n = K % GRAPH_STEPS
    tail = capture(tail_n, False) if tail_n else None
    reps = K // GRAPH_STEPS

    def timed_region():
        for _ in range(reps):
            full.replay()
        if tail is not None:
            tail.replay()

    # warm replays, then the timed region bracketed by barrier + sync
    with torch.cuda.stream(stream):
        full.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks:
        clocks.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        timed_region()
        ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop() if clocks else None
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # per-kernel durations from a separately captured, profiled graph
    pg = capture(GRAPH_STEPS, True)
    with torch.cuda.stream(stream):
        pg.replay()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        pg.replay()
    prof = ctx.profile_end()
    del pg, full, tail

    # end-to-end through the host-buffer entry point (pinned host memory)
    e2e_steps = min(K, 2048)
    h_logits = torch.randn((64, NE), dtype=torch.float32).pin_memory()
    h_x = torch.randn((64, HIDDEN), dtype=torch.float32).pin_memory()
    h_out = torch.empty((64, HIDDEN), dtype=torch.float32).pin_memory()
    for s in range(8):
        g, u, d = layers[s % nl]
        ctx.moe_decode_hostio(g, u, d, h_logits[s % 64].data_ptr(), h_x[s % 64].data_ptr(),
                              h_out[s % 64].data_ptr(), 1, HIDDEN, INTER, NE, TOPK)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        g, u, d = layers[s % nl]
        ctx.moe_decode_hostio(g, u, d, h_logits[s % 64].data_ptr(), h_x[s % 64].data_ptr(),
                              h_out[s % 64].data_ptr(), 1, HIDDEN, INTER, NE, TOPK)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())

    matvec = matvec_sweep(torch, ctx, stream) if (rank == 0 and args.matvec) else None
    lmh = lm_head_bench(torch, ctx, stream, rank, world, dist) if args.lm_head else None
    pf = prefill_bench(torch, ctx, stream, L, args.prefill_steps) if (rank == 0 and args.prefill) else None
    result = None
    if rank == 0:
        result = report(args, world, ms_max, prof, clk, e2e_steps, e2e_s, matvec, raw)
        result["lm_head"] = lmh
        result["prefill"] = pf
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return result


def matvec_sweep(torch, ctx, stream):
    """HBM throughput of the fused dequant-matvec per format on a matrix of
    >= 512 MB (4x L2) in the packed layout, plus single-call latency of
    config 0's 512 x 2048 Q4_K matvec with L2 flushed."""
    from qw6_b200 import synth as S
    hbm, _ = peaks()
    out = {}
    shapes = {S.Q4_K: 2048, S.Q5_K: 2048, S.Q6_K: 2048, S.IQ2_XXS: 2048, S.IQ2_S: 4096, S.IQ3_S: 2048}
    for q, cols in shapes.items():
        row_bytes = cols // 256 * S.BLOCK_BYTES[q]
        rows = ((512 << 20) // row_bytes + 15) // 16 * 16
        pb = ctx.packed_bytes(q, rows, cols)
        w = torch.randint(0, 256, (pb,), dtype=torch.uint8, device="cuda")
        x = torch.randn(cols, device="cuda")
        y = torch.empty(rows, device="cuda")
        torch.cuda.synchronize()
        for _ in range(3):
            ctx.matvec(q, w.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols)
        ctx.synchronize()
        n = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            ctx.matvec(q, w.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / n
        bytes_ = rows * row_bytes + cols * 4 + rows * 4
        out[S.QUANT_NAMES[q]] = {"shape": [rows, cols], "bytes": bytes_, "us": round(ms * 1e3, 2),
                                 "gbs": round(bytes_ / ms / 1e6, 1), "frac": round(bytes_ / ms / 1e6 / hbm, 3)}
        del w, x, y
    # config 0 single call, L2 flushed between calls
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    w0 = torch.randint(0, 256, (ctx.packed_bytes(S.Q4_K, 512, 2048),), dtype=torch.uint8, device="cuda")
    x0 = torch.randn(2048, device="cuda")
    y0 = torch.empty(512, device="cuda")
    lat = []
    torch.cuda.synchronize()
    for i in range(25):
        with torch.cuda.stream(stream):
            flush.fill_(i & 255)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ctx.matvec(S.Q4_K, w0.data_ptr(), x0.data_ptr(), y0.data_ptr(), 512, 2048)
        e1.record(stream)
        torch.cuda.synchronize()
        if i >= 5:
            lat.append(e0.elapsed_time(e1) * 1e3)
    out["c0_q4k_512x2048_latency_us"] = round(float(np.median(lat)), 2)
    return out


PREFILL_FLOPS = 2 * 4096 * TOPK * (2 * INTER * HIDDEN + HIDDEN * INTER) * 2 // 2  # 2 FLOP per MAC


def prefill_bench(torch, ctx, stream, L, steps):
    """Config 3 on one GPU: 4096 bf16 tokens through the 256-expert layer
    (Q4_K gate/up, Q6_K down) with the tcgen05 grouped GEMMs; tokens/s and
    dense bf16 TFLOP/s (206.2 GFLOP per step) against the measured peak."""
    from qw6_b200 import synth as S
    gate, up, down, logits, xbits = S.config3()
    packs, held = [], []
    for q, m, r, c in ((S.Q4_K, gate, INTER, HIDDEN), (S.Q4_K, up, INTER, HIDDEN), (S.Q6_K, down, HIDDEN, INTER)):
        pb = ctx.packed_bytes(q, r, c)
        raw = torch.from_numpy(m.reshape(-1)).cuda()
        pk = torch.empty(pb * NE, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ctx.pack(q, raw.data_ptr(), pk.data_ptr(), r, c, NE, m[0].nbytes, pb)
        ctx.synchronize()
        held.append(pk)
        packs.append(L.ExpertPack(q, pk.data_ptr(), pb))
    lg = torch.from_numpy(logits).cuda()
    x = torch.from_numpy(xbits.view(np.int16)).cuda()
    out = torch.empty((4096, HIDDEN), device="cuda")
    torch.cuda.synchronize()

    def one():
        ctx.moe_prefill(packs[0], packs[1], packs[2], lg.data_ptr(), x.data_ptr(), out.data_ptr(), 4096, HIDDEN,
                        INTER, NE, TOPK)

    for _ in range(3):
        one()
    ctx.check_device_errors()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        one()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    ctx.profile_begin(8 * 6)
    one()
    prof = ctx.profile_end()
    ctx.check_device_errors()
    pk_bf16 = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] if (
        ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    tflops = PREFILL_FLOPS / (ms / 1e3) / 1e12
    return {"workload": "config 3: 4096 tokens, 256 experts, top-8, bias N(0,0.5), 1 GPU",
            "steps": steps, "ms_per_step": round(ms, 4), "tokens_s": round(4096 / (ms / 1e3), 1),
            "tflops": round(tflops, 1), "frac_bf16_peak": round(tflops / pk_bf16, 3),
            "kernels": {k: {"avg_us": round(v[0] / v[1] * 1e3, 2), "launches": v[1]} for k, v in prof.items()}}


def lm_head_bench(torch, ctx, stream, rank, world, dist):
    """Config 4's Q6_K LM head [248320 x 2048] with fused argmax, row-sharded
    over the ranks (rank r holds rows [r*V/N, (r+1)*V/N)); the shards' 8-byte
    (logit, index) keys are all-gathered with NCCL and reduced on every rank.
    Returns per-token latency and tokens/s for batch 1 and batch 32."""
    from qw6_b200 import synth as S
    hbm, _ = peaks()
    V, H = S.VOCAB, HIDDEN
    r0 = (V * rank // world) // 16 * 16
    r1 = V if rank == world - 1 else (V * (rank + 1) // world) // 16 * 16
    rows = r1 - r0
    pb = ctx.packed_bytes(S.Q6_K, rows, H)
    w = torch.randint(0, 256, (pb,), dtype=torch.uint8, device="cuda")
    res = {}
    for ntok in (1, 32):
        x = torch.randn((ntok, H), device="cuda")
        keys = torch.zeros((ntok,), dtype=torch.int64, device="cuda")
        allk = torch.zeros((world, ntok), dtype=torch.int64, device="cuda")
        idx = torch.empty(ntok, dtype=torch.int32, device="cuda")
        val = torch.empty(ntok, dtype=torch.float32, device="cuda")

        def one():
            ctx.lm_head_argmax(S.Q6_K, w.data_ptr(), x.data_ptr(), ntok, rows, H, r0, keys.data_ptr())
            if world > 1:
                with torch.cuda.stream(stream):
                    dist.all_gather_into_tensor(allk.view(-1), keys)
                ctx.argmax_keys_reduce(allk.data_ptr(), world, ntok, idx.data_ptr(), val.data_ptr())
            else:
                ctx.argmax_keys_reduce(keys.data_ptr(), 1, ntok, idx.data_ptr(), val.data_ptr())

        for _ in range(3):
            one()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        n = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            one()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / n], device="cuda", dtype=torch.float64)
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        shard_bytes = rows * (H // 256) * 210 + ntok * H * 4
        res[f"b{ntok}"] = {"us_per_call": round(ms * 1e3, 2), "tokens_s": round(ntok / (ms / 1e3), 1),
                           "shard_rows": rows, "shard_gbs": round(shard_bytes / ms / 1e6, 1),
                           "shard_frac": round(shard_bytes / ms / 1e6 / hbm, 3)}
    res["shards"] = world
    res["collective"] = "NCCL all_gather of 8-byte keys" if world > 1 else None
    del w
    return res


def traffic_from_profiles(kernel: str):
    """dram bytes per launch recorded from an ncu capture in profiles/."""
    for p in sorted((ROOT / "profiles").glob("*.md")):
        for line in p.read_text().splitlines():
            if line.startswith(f"dram_bytes_per_launch[{kernel}]"):
                try:
                    return int(line.split("=")[1].split()[0])
                except (IndexError, ValueError):
                    return None
    return None


def report(args, world, ms_max, prof, clk, e2e_steps, e2e_s, matvec, raw):
    hbm, peak_kind = peaks()
    K = args.steps
    tokens = K * world
    value = tokens / (ms_max / 1e3)
    # roofline of the dominant kernel (largest total time)
    per_launch = {
        "moe_gateup": TOPK * 2 * Q4K_BYTES_EXPERT + HIDDEN * 4 + TOPK * INTER * 4,
        "moe_down": TOPK * Q6K_BYTES_EXPERT + TOPK * INTER * 4 + HIDDEN * 4,  # down + fused combine
    }
    dom = max((k for k in prof if k in per_launch), key=lambda k: prof[k][0])
    dom_ms = prof[dom][0] / prof[dom][1]
    achieved = per_launch[dom] / (dom_ms / 1e3) / 1e9
    traffic = traffic_from_profiles(dom)
    step_bytes = WEIGHT_BYTES_TOKEN + HIDDEN * 4 * 2 + NE * 4
    launches = sum(c for _, c in prof.values()) // GRAPH_STEPS * K
    kernels = {k: {"avg_us": round(v[0] / v[1] * 1e3, 2), "launches_profiled": v[1]} for k, v in prof.items()}

    cpu = None
    if args.cpu_baseline:
        gate, up, down = raw
        from qw6_b200 import synth as S
        _, _, _, lg, x = S.config1()
        rng = np.random.Generator(np.random.PCG64(77))
        lgs = np.concatenate([lg, rng.standard_normal((15, NE), dtype=np.float32)])
        xs = np.concatenate([x, rng.standard_normal((15, HIDDEN), dtype=np.float32)])
        rate, units, dt = cpu_reference_rate(gate, up, down, lgs, xs, budget_s=12.0, threads=1)
        cpu = {"value": round(rate, 3), "unit": "tokens/s", "cores": 1, "kind": "reference",
               "sample": f"{units} (token, expert) units = {units / TOPK:.1f} tokens of config 1 through qw6's own "
                         f"qw6_cpu_moe_route / qw6_tensor_matvec / qw6_silu (oracle/_ref), 1 thread, {dt:.1f} s"}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms_max / K, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "s8 mma (int32 acc) + f32", "data": "synthetic (seeded GGUF blocks, config 1)",
        "config": {"workload": "config 1: MoE FFN layer, decode batch 1", "hidden": HIDDEN, "experts": NE,
                   "top_k": TOPK, "inter": INTER, "gate_up": "Q4_K", "down": "Q6_K",
                   "parallelism": "replicas" if world > 1 else "1 GPU",
                   "l2": f"inputs larger than L2: {args.layers} resident layer copies "
                         f"({args.layers * NE * (2 * Q4K_BYTES_EXPERT + Q6K_BYTES_EXPERT) / 1e9:.1f} GB), "
                         f"step s uses layer s % {args.layers}",
                   "graph": f"CUDA graph of {GRAPH_STEPS} steps replayed"},
        "hbm_gbs_step": round(step_bytes * tokens / (ms_max / 1e3) / 1e9 / world, 1),
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 3), "peak_kind": peak_kind, "traffic": traffic,
                     "algorithmic_bytes_per_launch": per_launch[dom]},
        "kernels": kernels,
        "e2e": {"value": round(e2e_steps * world / e2e_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": (NE + HIDDEN) * 4, "d2h_bytes_per_step": HIDDEN * 4,
                "api": "qw6cu_moe_decode_hostio (pinned host logits/x/out, synchronous per step)"},
        "gpu_launches": int(launches),
        "clocks": clk,
        "cpu_baseline": cpu,
        "matvec": matvec,
    }
    return line


# --------------------------------------------------------- reference arm --

def run_reference(args, rank, world):
    if rank != 0:
        return None
    from qw6_b200 import synth as S
    gate, up, down, lg, x = S.config1()
    rng = np.random.Generator(np.random.PCG64(77))
    lgs = np.concatenate([lg, rng.standard_normal((63, NE), dtype=np.float32)])
    xs = np.concatenate([x, rng.standard_normal((63, HIDDEN), dtype=np.float32)])
    from oracle.oracle import Reference, cpu_count
    threads = cpu_count()
    # each step: `threads` (token, expert) units in parallel; bound the run to a few minutes
    from concurrent.futures import ThreadPoolExecutor
    ref = Reference()
    routes = [ref.moe_route(lgs[t], TOPK) for t in range(lgs.shape[0])]

    def unit(u):
        t, k = divmod(u, TOPK)
        t %= lgs.shape[0]
        e = int(routes[t][0][k])
        g = ref.matvec(4, gate[e], xs[t], INTER, HIDDEN)
        uu = ref.matvec(4, up[e], xs[t], INTER, HIDDEN)
        mid = np.array([ref.silu(float(v)) for v in g], np.float32) * uu
        return np.float32(routes[t][1][k]) * ref.matvec(7, down[e], mid.astype(np.float32), HIDDEN, INTER)

    K, W = args.steps, args.warmup
    with ThreadPoolExecutor(max_workers=threads) as ex:
        t_unit0 = time.perf_counter()
        list(ex.map(unit, range(threads)))
        t_unit = time.perf_counter() - t_unit0
        per_step = threads
        budget = 180.0
        if (K + W) * t_unit > budget:  # shrink the per-step sample to stay within a few minutes
            per_step = max(1, int(threads * budget / ((K + W) * t_unit)))
        done = 0
        for _ in range(W):
            list(ex.map(unit, range(done, done + per_step)))
            done += per_step
        t0 = time.perf_counter()
        for _ in range(K):
            list(ex.map(unit, range(done, done + per_step)))
            done += per_step
        dt = time.perf_counter() - t0
    value = K * per_step / TOPK / dt
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(dt / K * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF blocks, config 1)",
        "config": {"workload": "config 1: MoE FFN layer, decode batch 1", "hidden": HIDDEN, "experts": NE,
                   "top_k": TOPK, "inter": INTER, "gate_up": "Q4_K", "down": "Q6_K"},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": f"{per_step} (token, expert) units per step on {threads} threads through "
                                   "qw6's own CPU code (oracle/_ref: qw6_cpu_moe_route, qw6_tensor_matvec, "
                                   "qw6_silu); the reference's Vulkan path is unavailable on this box"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8192)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="resident layer copies (16 keeps the working set >> L2; fewer for profiling)")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-matvec", dest="matvec", action="store_false")
    ap.add_argument("--no-lm-head", dest="lm_head", action="store_false")
    ap.add_argument("--no-prefill", dest="prefill", action="store_false")
    ap.add_argument("--prefill-steps", type=int, default=20)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank, local_rank, world = dist_env()
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        line = run_ours(args, rank, local_rank, world)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
