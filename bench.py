#!/usr/bin/env python3
"""Benchmark of the quantized-matvec / MoE path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: one prefill MoE FFN layer
over 4096 bf16 tokens -- hidden 2048, 256 experts, top-8, expert
intermediate 512, Q4_K gate/up, Q6_K down, router logits fp32 ~ N(0,1) plus
a per-expert bias ~ N(0,0.5).  At N GPUs the experts are sharded 256/N per
GPU (placed by qw6_b200.ep.balance_experts on the routing counts of an
independent calibration batch) and the tokens 4096/N per GPU (strong
scaling: the job is always the same 4096 tokens); a step is route -> count
-> count exchange and plan -> dispatch of token rows into the owners'
memory over NVLink -> tcgen05 grouped GEMMs on each owner, whose down GEMM
writes each output row back into its source's memory -> slot-order combine
(qw6_b200.ep.PeerMoE, this library's own kernels, no host round trip).  N
resident copies of each GPU's expert shard (~522 MB per GPU, > 4x L2) are
used round robin, one per step.

Printed JSON line (rank 0): metric "MoE-layer tokens/s" (whole job), the
dominant kernel's tensor-core roofline, an end-to-end number with the
step's logits/x copied from pinned host memory and the output read back
every step, the CPU baseline (qw6's own CPU code on a sample of the same
tokens), clocks sampled during the timed region, and sub-results: decode
(config 1, batch 1, CUDA graph, HBM roofline), the per-format matvec sweep
and the row-sharded LM head (config 4).

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


def timed(torch, stream, dist, fn, nsteps):
    """Device time of nsteps calls of fn on `stream`, bracketed by barrier +
    synchronize, max over ranks (ms)."""
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for s in range(nsteps):
            fn(s)
        ev1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([ev0.elapsed_time(ev1)], device="cuda", dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


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
    head = ep_bench(args, torch, ctx, L, stream, rank, world, dist)
    dec = decode_bench(args, torch, ctx, L, stream, rank, world, dist) if args.decode else None
    matvec = matvec_sweep(torch, ctx, stream) if (rank == 0 and args.matvec) else None
    lmh = lm_head_bench(torch, ctx, stream, rank, world, dist) if args.lm_head else None
    result = None
    if rank == 0:
        result = report(args, world, head)
        result["decode"] = dec
        result["matvec"] = matvec
        result["lm_head"] = lmh
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return result


PF_FLOPS_ROW = {"pf_gemm1": 2 * 2 * INTER * HIDDEN, "pf_gemm2": 2 * HIDDEN * INTER}  # per routed row
T3 = 4096


def ep_bench(args, torch, ctx, L, stream, rank, world, dist):
    """Config 3 with the experts sharded over the ranks.  N=1: the
    single-GPU layer (qw6cu_moe_prefill); N>1: the peer-memory expert-parallel
    layer (qw6_b200.ep.PeerMoE: dispatch/combine kernels over NVLink, no
    host round trip).  Timed steps are replayed from CUDA graphs; one eager
    step is profiled per kernel; the end-to-end leg copies each step's
    inputs from pinned host memory and reads the output back."""
    from qw6_b200 import synth as S
    from qw6_b200.ep import PeerMoE, balance_experts
    gate, up, down, logits, xbits, bias = S.config3(with_bias=True)
    epr, tpr = NE // world, T3 // world
    placement = None
    if world > 1:  # balance the ranks' rows on routing statistics of an independent calibration batch
        cal = S.router_sample(bias, T3, seed=1003)
        cnt = np.bincount(np.argsort(-cal, axis=1, kind="stable")[:, :TOPK].ravel(), minlength=NE)
        placement = balance_experts(cnt, world)
    mine_ids = placement[rank] if placement is not None else np.arange(rank * epr, (rank + 1) * epr)
    ncopies = world  # world copies of a 256/world-expert shard: ~522 MB resident per GPU
    copies = []
    for q, m, r, c in ((S.Q4_K, gate, INTER, HIDDEN), (S.Q4_K, up, INTER, HIDDEN), (S.Q6_K, down, HIDDEN, INTER)):
        mine = np.ascontiguousarray(m[mine_ids])
        pb = ctx.packed_bytes(q, r, c)
        raw = torch.from_numpy(mine.reshape(-1)).cuda()
        pk = torch.empty(pb * epr, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ctx.pack(q, raw.data_ptr(), pk.data_ptr(), r, c, epr, mine[0].nbytes, pb)
        ctx.synchronize()
        del raw
        copies.append((q, pb, [pk] + [pk.clone() for _ in range(ncopies - 1)]))
    packs = [tuple(L.ExpertPack(q, cp[i].data_ptr(), pb) for q, pb, cp in copies) for i in range(ncopies)]
    sl = slice(rank * tpr, (rank + 1) * tpr)
    lg = torch.from_numpy(logits[sl]).cuda()
    x = torch.from_numpy(xbits[sl].view(np.int16)).cuda()
    out = torch.empty((tpr, HIDDEN), dtype=torch.float32, device="cuda")
    pm = PeerMoE(ctx, *packs[0], NE, TOPK, HIDDEN, INTER, tpr, placement=placement) if world > 1 else None
    torch.cuda.synchronize()

    def step(s, lgt=lg, xt=x, o=out):
        pk = packs[s % ncopies]
        if pm is not None:
            pm(lgt, xt, o, packs=pk)
        else:
            ctx.set_stream(torch.cuda.current_stream().cuda_stream)
            ctx.moe_prefill(*pk, lgt.data_ptr(), xt.data_ptr(), o.data_ptr(), tpr, HIDDEN, INTER, NE, TOPK)

    K, W = args.steps, args.warmup
    with torch.cuda.stream(stream):
        for s in range(W):
            step(s)
    torch.cuda.synchronize()
    ctx.check_device_errors()

    G = max(1, min(K, 2 * ncopies if ncopies > 1 else 8))

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for s in range(n):
                step(s)
        return g

    full = capture(G)
    tail = capture(K % G) if K % G else None
    with torch.cuda.stream(stream):
        full.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank_of(rank)) if rank == 0 else None
    if clocks:
        clocks.start()
    reps = K // G
    ms = timed(torch, stream, dist, lambda i: (full if i < reps else tail).replay(), reps + (1 if tail else 0))
    clk = clocks.stop() if clocks else None
    ctx.check_device_errors()
    del full, tail

    # per-kernel device time from a separately captured graph of G steps
    # (event nodes around every launch), replayed twice; per-step averages
    ctx.profile_begin(32 * G + 8)
    pg = capture(G)
    for _ in range(2):
        with torch.cuda.stream(stream):
            pg.replay()
        torch.cuda.synchronize()
    prof = {k: (ms_ / G, n // G) for k, (ms_, n) in ctx.profile_end().items()}
    del pg
    rows = pm.last_rows() if pm is not None else tpr * TOPK

    # end to end: this step's logits/x from pinned host memory, output read back
    h_lg = torch.from_numpy(logits[sl]).pin_memory()
    h_x = torch.from_numpy(xbits[sl].view(np.int16)).pin_memory()
    h_out = torch.empty((tpr, HIDDEN), dtype=torch.float32).pin_memory()
    d_lg, d_x, d_out = torch.empty_like(lg), torch.empty_like(x), torch.empty_like(out)

    def e2e_step(s):
        d_lg.copy_(h_lg, non_blocking=True)
        d_x.copy_(h_x, non_blocking=True)
        step(s, d_lg, d_x, d_out)
        h_out.copy_(d_out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    with torch.cuda.stream(stream):
        for s in range(3):
            e2e_step(s)
    ke = max(1, min(K, 100))
    e2e_ms = timed(torch, stream, dist, e2e_step, ke)
    ctx.check_device_errors()
    out_ok = bool(np.isfinite(h_out.numpy()).all())
    if pm is not None:
        if dist:
            dist.barrier()
        pm.close()
    del packs, copies
    torch.cuda.empty_cache()
    return {"ms": ms, "clk": clk, "prof": prof, "rows": rows, "e2e_ms": e2e_ms, "e2e_steps": ke, "graph_steps": G,
            "h2d": tpr * NE * 4 + tpr * HIDDEN * 2, "d2h": tpr * HIDDEN * 4, "finite": out_ok,
            "cpu_data": (gate, up, down, logits[:16], S.bf16_to_f32(xbits[:16]))}


def local_rank_of(rank):
    return int(os.environ.get("LOCAL_RANK", rank))


def decode_bench(args, torch, ctx, L, stream, rank, world, dist):
    """Config 1 (decode batch 1) as N replicas: a CUDA graph of 256 steps
    replayed back to back over 16 resident layer copies; HBM roofline of
    the dominant kernel; end to end through qw6cu_moe_decode_hostio."""
    raw, packs, layers = build_layers(torch, ctx, L, args.layers)
    nl = args.layers
    K = args.decode_steps
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

    with torch.cuda.stream(stream):
        for s in range(max(args.warmup, 1)):
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
    reps = max(1, K // GRAPH_STEPS)
    K = reps * GRAPH_STEPS
    with torch.cuda.stream(stream):
        full.replay()
    torch.cuda.synchronize()
    ms = timed(torch, stream, dist, lambda s: full.replay(), reps)
    pg = capture(GRAPH_STEPS, True)
    with torch.cuda.stream(stream):
        pg.replay()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        pg.replay()
    prof = ctx.profile_end()
    del pg, full

    e2e_steps = min(K, 2048)
    h_logits = torch.randn((64, NE), dtype=torch.float32).pin_memory()
    h_x = torch.randn((64, HIDDEN), dtype=torch.float32).pin_memory()
    h_out = torch.empty((64, HIDDEN), dtype=torch.float32).pin_memory()

    def hostio(s):
        g, u, d = layers[s % nl]
        ctx.moe_decode_hostio(g, u, d, h_logits[s % 64].data_ptr(), h_x[s % 64].data_ptr(),
                              h_out[s % 64].data_ptr(), 1, HIDDEN, INTER, NE, TOPK)

    for s in range(8):
        hostio(s)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        hostio(s)
    te = torch.tensor([time.perf_counter() - t0], device="cuda", dtype=torch.float64)
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())
    del layers, packs
    torch.cuda.empty_cache()

    hbm, peak_kind = peaks()
    per_launch = {
        "moe_gateup": TOPK * 2 * Q4K_BYTES_EXPERT + HIDDEN * 4 + TOPK * INTER * 4,
        "moe_down": TOPK * Q6K_BYTES_EXPERT + TOPK * INTER * 4 + HIDDEN * 4,  # down + fused combine
    }
    dom = max((k for k in prof if k in per_launch), key=lambda k: prof[k][0])
    dom_ms = prof[dom][0] / prof[dom][1]
    achieved = per_launch[dom] / (dom_ms / 1e3) / 1e9
    step_bytes = WEIGHT_BYTES_TOKEN + HIDDEN * 4 * 2 + NE * 4
    tokens = K * world
    return {
        "workload": "config 1: MoE FFN layer, decode batch 1 (N independent replicas)",
        "tokens_s": round(tokens / (ms / 1e3), 1), "ms_per_step": round(ms / K, 5), "steps": K,
        "hbm_gbs_step": round(step_bytes * K / (ms / 1e3) / 1e9, 1),
        "l2": f"inputs larger than L2: {nl} resident layer copies "
              f"({nl * NE * (2 * Q4K_BYTES_EXPERT + Q6K_BYTES_EXPERT) / 1e9:.1f} GB), step s uses layer s % {nl}",
        "graph": f"CUDA graph of {GRAPH_STEPS} steps replayed",
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 3), "peak_kind": peak_kind,
                     "traffic": traffic_from_profiles(dom), "algorithmic_bytes_per_launch": per_launch[dom]},
        "kernels": {k: {"avg_us": round(v[0] / v[1] * 1e3, 2), "launches_profiled": v[1]} for k, v in prof.items()},
        "e2e": {"value": round(e2e_steps * world / e2e_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": (NE + HIDDEN) * 4, "d2h_bytes_per_step": HIDDEN * 4,
                "api": "qw6cu_moe_decode_hostio (pinned host logits/x/out, synchronous per step)"},
        "gpu_launches_per_step": sum(c for _, c in prof.values()) // GRAPH_STEPS,
    }


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


def bf16_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback (burst)"


def report(args, world, head):
    hbm, hbm_kind = peaks()
    tflops_peak, tf_kind = bf16_peak()
    K = args.steps
    ms = head["ms"]
    value = T3 * K / (ms / 1e3)
    prof, rows = head["prof"], head["rows"]
    dom = max((k for k in prof if k in PF_FLOPS_ROW), key=lambda k: prof[k][0])
    dom_ms = prof[dom][0] / prof[dom][1]
    flops = rows * PF_FLOPS_ROW[dom]
    achieved = flops / (dom_ms / 1e3) / 1e12
    launches = sum(c for _, c in prof.values())
    shard_weight_bytes = NE // world * (2 * Q4K_BYTES_EXPERT + Q6K_BYTES_EXPERT)
    cpu = None
    if args.cpu_baseline and world == 1:
        gate, up, down, lg, x = head["cpu_data"]
        rate, units, dt = cpu_reference_rate(gate, up, down, lg, x, budget_s=12.0, threads=1)
        cpu = {"value": round(rate, 3), "unit": "tokens/s", "cores": 1, "kind": "reference",
               "sample": f"{units} (token, expert) units = {units / TOPK:.1f} of config 3's tokens through qw6's own "
                         f"qw6_cpu_moe_route / qw6_tensor_matvec / qw6_silu (oracle/_ref), 1 thread, {dt:.1f} s"}
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16 (tcgen05 kind::f16, f32 accumulate; Q4_K/Q6_K weights)",
        "data": "synthetic (seeded GGUF blocks, config 3)",
        "config": {"workload": "config 3: prefill MoE FFN layer, 4096 tokens", "tokens": T3, "hidden": HIDDEN,
                   "experts": NE, "top_k": TOPK, "inter": INTER, "gate_up": "Q4_K", "down": "Q6_K",
                   "router_bias": "N(0,0.5) per expert",
                   "parallelism": f"ep{world}: {NE // world} experts and {T3 // world} tokens per GPU"
                                  + (", dispatch/combine by this library's kernels over NVLink peer memory, "
                                     "experts placed by balance_experts on the routing counts of an independent "
                                     "calibration batch (same router bias, fresh token noise)"
                                     if world > 1 else ""),
                   "graph": f"CUDA graphs of {head['graph_steps']} steps replayed",
                   "l2": f"inputs larger than L2: {world} resident copies of each GPU's expert shard "
                         f"({world * shard_weight_bytes / 1e6:.0f} MB per GPU), step s uses copy s % {world}"},
        "roofline": {"bound": "tensor", "kernel": dom, "achieved": round(achieved, 1), "peak": tflops_peak,
                     "unit": "TFLOP/s", "frac": round(achieved / tflops_peak, 3), "peak_kind": tf_kind,
                     "traffic": traffic_from_profiles(dom) if world == 1 else None,
                     "algorithmic_flops_per_launch": flops, "rows_rank0": rows},
        "hbm": {"weight_bytes_per_step": shard_weight_bytes, "gbs": round(shard_weight_bytes * K / (ms / 1e3) / 1e9, 1),
                "frac": round(shard_weight_bytes * K / (ms / 1e3) / 1e9 / hbm, 4), "peak": hbm, "peak_kind": hbm_kind},
        "kernels": {k: {"avg_us": round(v[0] / v[1] * 1e3, 2), "launches_per_step": v[1]} for k, v in prof.items()},
        "e2e": {"value": round(T3 * head["e2e_steps"] / (head["e2e_ms"] / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": head["h2d"], "d2h_bytes_per_step": head["d2h"],
                "api": ("qw6_b200.ep.PeerMoE" if world > 1 else "qw6cu_moe_prefill")
                       + " with this rank's logits/x copied from pinned host memory and the fp32 output copied "
                         "back and synchronized every step (per-rank bytes)",
                "output_finite": head["finite"]},
        "gpu_launches": int(launches * K),
        "clocks": head["clk"],
        "cpu_baseline": cpu,
    }


# --------------------------------------------------------- reference arm --

def run_reference(args, rank, world):
    if rank != 0:
        return None
    from qw6_b200 import synth as S
    gate, up, down, lg, xb = S.config3()
    lgs, xs = lg[:256], S.bf16_to_f32(xb[:256])
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
        "warmup": W, "ms_per_step": round(dt / K * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF blocks, config 3)",
        "config": {"workload": "config 3: prefill MoE FFN layer, 4096 tokens", "tokens": T3, "hidden": HIDDEN,
                   "experts": NE, "top_k": TOPK, "inter": INTER, "gate_up": "Q4_K", "down": "Q6_K",
                   "router_bias": "N(0,0.5) per expert"},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": f"{per_step} (token, expert) units per step of config 3's first 256 tokens on "
                                   f"{threads} threads through qw6's own CPU code (oracle/_ref: qw6_cpu_moe_route, "
                                   "qw6_tensor_matvec, qw6_silu; the reference has no batched path, so tokens are "
                                   "looped as qw6_prefill does); the reference's Vulkan path is unavailable on "
                                   "this box"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="resident layer copies (16 keeps the working set >> L2; fewer for profiling)")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-matvec", dest="matvec", action="store_false")
    ap.add_argument("--no-lm-head", dest="lm_head", action="store_false")
    ap.add_argument("--no-decode", dest="decode", action="store_false")
    ap.add_argument("--decode-steps", type=int, default=8192)
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
