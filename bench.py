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
#
# qw6's own CPU implementation of the layer (oracle/_ref, compiled from the
# reference sources): qw6_cpu_moe_route + the expert loop of
# qw6_apply_layer_moe (qw6.c:2246-2264), run entirely in C per token
# (ref_moe_tokens).  qw6 is single-threaded; the harness slices tokens over a
# fork pool of one process per host core.  The pool is forked before this
# process touches CUDA (a pool forked after CUDA initialisation can hang).

_POOL = {}  # set in the parent before forking; the workers inherit it


def host_info() -> dict:
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    from oracle.oracle import cpu_count
    return {"nproc": os.cpu_count(), "usable_cores": cpu_count(), "cpu_model": model}


def _pool_tokens(span):
    t0, t1 = span
    ref = _POOL.get("ref")
    if ref is None:
        from oracle.oracle import Reference
        ref = _POOL["ref"] = Reference()
    gate, up, down, logits, x = _POOL["data"]
    ref.moe_tokens(4, gate, up, 7, down, logits, x, t0, t1, top_k=TOPK)
    return t1 - t0


class CpuMoE:
    """qw6's CPU MoE layer over a token sample, 1 thread or a fork pool."""

    def __init__(self, gate, up, down, logits, x, workers: int):
        _POOL["data"] = (gate, up, down, logits, x)
        self.ntok = logits.shape[0]
        self.workers = workers
        self.next = 0
        self.pool = None
        if workers > 1:
            import multiprocessing as mp
            self.pool = mp.get_context("fork").Pool(workers)

    def spans(self, ntok, per):
        out = []
        while ntok > 0:
            n = min(per, ntok, self.ntok - self.next)
            out.append((self.next, self.next + n))
            self.next = (self.next + n) % self.ntok
            ntok -= n
        return out

    def run(self, ntok, per=1) -> float:
        """Seconds to run ntok tokens of the sample (continuing round robin)."""
        sp = self.spans(ntok, per)
        t0 = time.perf_counter()
        if self.pool is None:
            for s in sp:
                _pool_tokens(s)
        else:
            self.pool.map(_pool_tokens, sp, chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        if self.pool is not None:
            self.pool.close()
            self.pool.join()
            self.pool = None


def cpu_baseline_c3(gate, up, down, logits, x, seconds_1=4.0, seconds_n=10.0) -> dict:
    """qw6's CPU path on config 3's tokens: ~seconds_1 on one thread and
    ~seconds_n over all usable cores (token-sliced fork pool)."""
    from oracle.oracle import cpu_count
    info = host_info()
    one = CpuMoE(gate, up, down, logits, x, 1)
    one.run(1)  # warm (loads the library, touches the first experts)
    n1, dt1 = 0, 0.0
    while dt1 < seconds_1:
        dt1 += one.run(2)
        n1 += 2
    rate1 = n1 / dt1
    workers = cpu_count()
    pool = CpuMoE(gate, up, down, logits, x, workers)
    pool.run(workers)
    per_round = workers * max(1, int(rate1 * 2.0))  # ~2 s rounds
    nn, dtn = 0, 0.0
    while dtn < seconds_n:
        dtn += pool.run(per_round)
        nn += per_round
    pool.close()
    raten = nn / dtn
    return {"value": round(raten, 2), "unit": "tokens/s", "cores": workers, "kind": "reference",
            "value_1core": round(rate1, 2),
            "sample": f"{nn} of config 3's tokens in {dtn:.1f} s over a fork pool of {workers} processes (token "
                      f"slices; 'harness parallelised', qw6 itself is single-threaded) and {n1} tokens in "
                      f"{dt1:.1f} s on 1 thread, each token through qw6's own qw6_cpu_moe_route and expert loop "
                      "(qw6_tensor_matvec, qw6_silu; qw6.c:2246-2264) compiled from the reference sources "
                      "(oracle/_ref); the reference's Vulkan path is unavailable on this box",
            "host": info}


# ------------------------------------------------------------- our arm ----

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

    from qw6_b200 import synth as S
    c3 = S.config3(with_bias=True)
    cpu = None
    if args.cpu_baseline and world == 1 and rank == 0:
        # before this process initialises CUDA: the pool is forked
        gate, up, down, logits, xbits, _ = c3
        cpu = cpu_baseline_c3(gate, up, down, logits, S.bf16_to_f32(xbits))

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
    head = ep_bench(args, torch, ctx, L, stream, rank, world, dist, c3)
    del c3
    dec = {}
    if args.decode:
        for c in (1, 2):
            dec[f"config{c}"] = moe_decode_bench(args, torch, ctx, L, stream, rank, world, dist, c)
    matvec = None
    if rank == 0 and args.matvec:
        matvec = {"configs": matvec_configs(torch, ctx, stream), "tall_sweep": matvec_sweep(torch, ctx, stream)}
    lmh = lm_head_bench(torch, ctx, stream, rank, world, dist) if args.lm_head else None
    dstep = decoder_bench(args, ctx, L) if (args.decoder and rank == 0) else None
    if dist:
        dist.barrier()
    result = None
    if rank == 0:
        result = report(args, world, head, cpu)
        result["decode"] = dec or None
        result["matvec"] = matvec
        result["lm_head"] = lmh
        result["decoder"] = dstep
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return result


PF_FLOPS_ROW = {"pf_gemm1": 2 * 2 * INTER * HIDDEN, "pf_gemm2": 2 * HIDDEN * INTER}  # per routed row
T3 = 4096


def ep_bench(args, torch, ctx, L, stream, rank, world, dist, c3):
    """Config 3 with the experts sharded over the ranks.  N=1: the
    single-GPU layer (qw6cu_moe_prefill); N>1: the peer-memory expert-parallel
    layer (qw6_b200.ep.PeerMoE: dispatch/combine kernels over NVLink, no
    host round trip).  Timed steps are replayed from CUDA graphs; one eager
    step is profiled per kernel; the end-to-end leg copies each step's
    inputs from pinned host memory and reads the output back."""
    from qw6_b200 import synth as S
    from qw6_b200.ep import PeerMoE, balance_experts
    gate, up, down, logits, xbits, bias = c3
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

    # end to end: every step copies its logits/x in from pinned host memory
    # and reads its output back, pipelined over two device slots (copy-in of
    # step s+1 and read-back of step s-1 beside the experts of step s): one
    # call of the C ABI's host-buffer entry point over all ke steps
    # (qw6cu_moe_prefill_hostio; N>1 qw6cu_ep_layer_hostio on every rank).
    host_cpus = bind_host_near_gpu(torch, torch.cuda.current_device())
    nh = 4  # distinct page-locked host batches, used in turn
    h_lg = [torch.from_numpy(logits[sl]).pin_memory() for _ in range(nh)]
    h_x = [torch.from_numpy(xbits[sl].view(np.int16)).pin_memory() for _ in range(nh)]
    h_outs = [torch.empty((tpr, HIDDEN), dtype=torch.float32).pin_memory() for _ in range(nh)]
    ke = 128  # enough steps that filling and draining the pipeline (one copy-in, one read-back) is ~1%

    def e2e_run(n):
        lgp, xp, op = ([h[s % nh].data_ptr() for s in range(n)] for h in (h_lg, h_x, h_outs))
        if pm is None:
            ctx.set_stream(stream.cuda_stream)
            ctx.moe_prefill_hostio(*packs[0], lgp, xp, op, tpr, HIDDEN, INTER, NE, TOPK)
        else:
            pm.hostio(lgp, xp, op, tpr, packs=packs[0])

    with torch.cuda.stream(stream):
        e2e_run(3)
    torch.cuda.synchronize()
    # three timed calls of ke steps each, the median reported: host<->device
    # copy rates on these shared hosts vary from one call to the next
    e2e_runs = [timed(torch, stream, dist, lambda i: e2e_run(ke), 1) for _ in range(3)]
    e2e_ms = float(np.median(e2e_runs))
    ctx.check_device_errors()
    h_out = h_outs[(ke - 1) % nh]
    out_ok = bool(np.isfinite(h_out.numpy()).all())
    # the device-resident steps ran the same inputs through the same weights
    same = bool(np.array_equal(h_out.numpy().view(np.uint32), out.cpu().numpy().view(np.uint32)))
    if pm is not None:
        if dist:
            dist.barrier()
        pm.close()
    del packs, copies
    torch.cuda.empty_cache()
    return {"ms": ms, "clk": clk, "prof": prof, "rows": rows, "e2e_ms": e2e_ms, "e2e_runs_ms": e2e_runs,
            "e2e_steps": ke, "graph_steps": G,
            "h2d": tpr * NE * 4 + tpr * HIDDEN * 2, "d2h": tpr * HIDDEN * 4, "finite": out_ok, "same": same,
            "host_cpus": len(host_cpus) if host_cpus else None}


def local_rank_of(rank):
    return int(os.environ.get("LOCAL_RANK", rank))


def bind_host_near_gpu(torch, device):
    """Run this thread on the CPUs of the GPU's PCIe root (sysfs local_cpulist
    of the device), so that page-locked buffers allocated afterwards come from
    that NUMA node's memory: host<->device copies from the other socket's
    memory run at about half the rate.  Returns the CPU list, or None when
    sysfs does not say."""
    p = torch.cuda.get_device_properties(device)
    path = Path(f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0/local_cpulist")
    try:
        cpus = set()
        for part in path.read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return sorted(cpus)
    except (OSError, ValueError):
        return None


IQ2XXS_BYTES_EXPERT = 512 * 8 * 66                            # one IQ2_XXS expert matrix (gate, up or down)
DECODE = {  # config: (tokens, gate/up quant, down quant, gate/up bytes per expert, down bytes per expert, graph steps)
    1: (1, 4, 7, Q4K_BYTES_EXPERT, Q6K_BYTES_EXPERT, 256),
    2: (64, 13, 13, IQ2XXS_BYTES_EXPERT, IQ2XXS_BYTES_EXPERT, 32),
}


def distinct_experts(logits: np.ndarray) -> int:
    """Experts a batch of router logits selects (top-8, lower index on ties,
    as qw6_cpu_moe_route)."""
    return int(np.unique(np.argsort(-logits, axis=1, kind="stable")[:, :TOPK]).size)


def moe_decode_bench(args, torch, ctx, L, stream, rank, world, dist, config):
    """Configs 1 and 2 (decode batch 1 / batched decode of 64 tokens with
    IQ2_XXS experts) as N replicas: a CUDA graph of steps replayed back to
    back over `args.layers` resident layer copies (step s uses copy s % layers
    and router/activation slot s % 16); HBM roofline of the step and of its
    dominant kernel over the distinct experts' bytes; end to end through
    qw6cu_moe_decode_hostio."""
    from qw6_b200 import synth as S
    ntok, gq, dq, gub, dnb, gsteps = DECODE[config]
    nl, nslots = args.layers, 16
    rng = np.random.Generator(np.random.PCG64(config))
    gate, up, down = S.moe_weights(rng, NE, gq, dq)
    copies = []
    for q, m, r, c in ((gq, gate, INTER, HIDDEN), (gq, up, INTER, HIDDEN), (dq, down, HIDDEN, INTER)):
        pb = ctx.packed_bytes(q, r, c)
        raw = torch.from_numpy(m.reshape(-1)).cuda()
        pk = torch.empty(pb * NE, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ctx.pack(q, raw.data_ptr(), pk.data_ptr(), r, c, NE, m[0].nbytes, pb)
        ctx.synchronize()
        del raw
        copies.append((q, pb, [pk] + [pk.clone() for _ in range(nl - 1)]))
    del gate, up, down
    layers = [tuple(L.ExpertPack(q, cp[i].data_ptr(), pb) for q, pb, cp in copies) for i in range(nl)]
    # router logits and activations of 16 token batches (seeded, N(0,1))
    lg_np = [np.random.Generator(np.random.PCG64(1000 * config + 17 * rank + j)).standard_normal(
        (ntok, NE), dtype=np.float32) for j in range(nslots)]
    eact = [distinct_experts(v) for v in lg_np]
    logits = torch.from_numpy(np.stack(lg_np)).cuda()
    xs = torch.from_numpy(np.random.Generator(np.random.PCG64(2000 * config + rank)).standard_normal(
        (nslots, ntok, HIDDEN), dtype=np.float32)).cuda()
    outs = torch.empty((nslots, ntok, HIDDEN), device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()

    def step(s):
        g, u, d = layers[s % nl]
        j = s % nslots
        ctx.moe_decode(g, u, d, logits[j].data_ptr(), xs[j].data_ptr(), outs[j].data_ptr(), ntok, HIDDEN, INTER,
                       NE, TOPK)

    with torch.cuda.stream(stream):
        for s in range(max(args.warmup, 3)):
            step(s)
    ctx.synchronize()
    ctx.check_device_errors()

    def capture(nsteps, profile):
        g = torch.cuda.CUDAGraph()
        if profile:
            ctx.profile_begin(8 * nsteps + 8)
        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
            for s in range(nsteps):
                step(s)
        return g

    K = args.decode_steps if config == 1 else max(gsteps, args.decode_steps // 8)
    full = capture(gsteps, False)
    reps = max(1, K // gsteps)
    K = reps * gsteps
    with torch.cuda.stream(stream):
        full.replay()
    torch.cuda.synchronize()
    ms = timed(torch, stream, dist, lambda s: full.replay(), reps)
    pg = capture(gsteps, True)
    for _ in range(2):
        with torch.cuda.stream(stream):
            pg.replay()
        torch.cuda.synchronize()
    prof = ctx.profile_end()
    del pg, full
    ctx.check_device_errors()

    # end to end: host logits/x in, host out, synchronous per step
    e2e_steps = min(K, 2048 if config == 1 else 256)
    h_logits = torch.from_numpy(np.stack(lg_np)).pin_memory()
    h_x = xs.cpu().pin_memory()
    h_out = torch.empty((nslots, ntok, HIDDEN), dtype=torch.float32).pin_memory()

    def hostio(s):
        g, u, d = layers[s % nl]
        j = s % nslots
        ctx.moe_decode_hostio(g, u, d, h_logits[j].data_ptr(), h_x[j].data_ptr(), h_out[j].data_ptr(), ntok,
                              HIDDEN, INTER, NE, TOPK)

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
    del layers, copies
    torch.cuda.empty_cache()

    hbm, peak_kind = peaks()
    ea = float(np.mean([eact[s % nslots] for s in range(K)]))
    xb, ob, lb = ntok * HIDDEN * 4, ntok * HIDDEN * 4, ntok * NE * 4
    mid = ntok * TOPK * INTER * 4
    per_launch = {"moe_gateup": ea * 2 * gub + xb + mid, "moe_down": ea * dnb + mid + ob}
    if config == 1:  # down + fused combine; gate/up routes itself
        per_launch["moe_gateup"] += lb
    else:
        per_launch["moe_down"] = ea * dnb + mid + ntok * TOPK * HIDDEN * 4
    step_bytes = ea * (2 * gub + dnb) + xb + ob + lb
    dom = max((k for k in prof if k in per_launch), key=lambda k: prof[k][0])
    dom_ms = prof[dom][0] / prof[dom][1]
    achieved = per_launch[dom] / (dom_ms / 1e3) / 1e9
    step_gbs = step_bytes * K / (ms / 1e3) / 1e9
    tokens = K * ntok * world
    return {
        "workload": {1: "config 1: MoE FFN layer, decode batch 1, Q4_K gate/up + Q6_K down",
                     2: "config 2: batched-decode MoE layer, 64 tokens, IQ2_XXS gate/up/down"}[config]
                    + " (N independent replicas)",
        "tokens_s": round(tokens / (ms / 1e3), 1), "ms_per_step": round(ms / K, 5), "steps": K,
        "distinct_experts_per_step": round(ea, 2),
        "algorithmic_bytes_per_step": int(step_bytes),
        "hbm_gbs_step": round(step_gbs, 1), "hbm_frac_step": round(step_gbs / hbm, 3),
        "l2": f"inputs larger than L2: {nl} resident layer copies "
              f"({nl * NE * (2 * gub + dnb) / 1e9:.1f} GB), step s uses layer s % {nl}",
        "graph": f"CUDA graph of {gsteps} steps replayed",
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 3), "peak_kind": peak_kind,
                     "traffic": traffic_from_profiles(f"decode_c{config}_{dom}"),
                     "algorithmic_bytes_per_launch": int(per_launch[dom])},
        "kernels": {k: {"avg_us": round(v[0] / v[1] * 1e3, 2), "launches_profiled": v[1]} for k, v in prof.items()},
        "e2e": {"value": round(e2e_steps * ntok * world / e2e_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": lb + xb, "d2h_bytes_per_step": ob,
                "api": "qw6cu_moe_decode_hostio (pinned host logits/x/out, synchronous per step)"},
        "gpu_launches_per_step": sum(c for _, c in prof.values()) // gsteps,
    }


MATVEC_CONFIGS = (  # (name, quant, rows, cols): config 0 and config 4's projections
    ("c0_q4k_512x2048", 4, 512, 2048),
    ("c4_q5k_4096x2048", 6, 4096, 2048),
    ("c4_iq2s_2048x4096", 11, 2048, 4096),
    ("c4_iq3s_2048x2048", 9, 2048, 2048),
)


def matvec_configs(torch, ctx, stream):
    """Configs 0 and 4 (projections) at their own shapes, batch 1 and 32, by
    the rotation protocol: K distinct copies of the packed matrix (K x bytes
    >= 512 MB, 4x L2) launched back to back inside one CUDA graph, median of
    >= 20 replays; plus the single-call latency with L2 flushed."""
    from qw6_b200 import synth as S
    hbm, kind = peaks()
    rng = np.random.Generator(np.random.PCG64(4))
    res = {"protocol": "K copies (K x weight bytes >= 512 MB) rotated in one CUDA graph; median of 25 replays",
           "peak": hbm, "peak_kind": kind}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for name, q, rows, cols in MATVEC_CONFIGS:
        raw = S.make_matrix(q, rows, cols, rng) if q != 4 else S.config0()[0]
        pb = ctx.packed_bytes(q, rows, cols)
        stride = (pb + 255) // 256 * 256
        ncopy = max(1, -(-(512 << 20) // pb))
        w = torch.empty(stride * ncopy, dtype=torch.uint8, device="cuda")
        rd = torch.from_numpy(raw.reshape(-1)).cuda()
        torch.cuda.synchronize()
        ctx.pack(q, rd.data_ptr(), w.data_ptr(), rows, cols)
        ctx.synchronize()
        w.view(ncopy, stride)[1:] = w.view(ncopy, stride)[0]
        del rd
        wbytes = rows * (cols // 256) * S.BLOCK_BYTES[q]
        entry = {"shape": [rows, cols], "weight_bytes": wbytes, "copies": ncopy}
        for ntok in (1, 32):
            x = torch.randn(ntok, cols, device="cuda")
            y = torch.empty(ntok, rows, device="cuda")
            torch.cuda.synchronize()
            for _ in range(3):
                ctx.matvec(q, w.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, ntok)
            ctx.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                for i in range(ncopy):
                    ctx.matvec(q, w.data_ptr() + i * stride, x.data_ptr(), y.data_ptr(), rows, cols, ntok)
            with torch.cuda.stream(stream):
                g.replay()
            torch.cuda.synchronize()
            times = []
            for _ in range(25):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                with torch.cuda.stream(stream):
                    g.replay()
                e1.record(stream)
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1) / ncopy)
            ms = float(np.median(times))
            del g
            # single call with L2 flushed
            lat = []
            for i in range(12):
                with torch.cuda.stream(stream):
                    flush.fill_(i & 255)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                ctx.matvec(q, w.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, ntok)
                e1.record(stream)
                torch.cuda.synchronize()
                if i >= 2:
                    lat.append(e0.elapsed_time(e1) * 1e3)
            b = wbytes + ntok * cols * 4 + ntok * rows * 4
            entry[f"b{ntok}"] = {"us_per_call": round(ms * 1e3, 3), "gbs": round(b / ms / 1e6, 1),
                                 "frac": round(b / ms / 1e6 / hbm, 3),
                                 "single_call_l2_flushed_us": round(float(np.median(lat)), 2)}
            del x, y
        res[name] = entry
        del w
        torch.cuda.empty_cache()
    del flush
    return res


def matvec_sweep(torch, ctx, stream):
    """Streaming HBM throughput of the fused dequant-matvec per format, batch
    1, on one tall matrix of >= 512 MB (4x L2) in the packed layout, 20
    launches back to back."""
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
    return out


def lm_head_bench(torch, ctx, stream, rank, world, dist):
    """Config 4's Q6_K LM head [248320 x 2048] with fused argmax, row-sharded
    over the ranks (qw6_b200.lm_head: rank r holds shard_rows(V, N, r)); the
    shards' 8-byte (logit, index) keys are all-gathered with NCCL and reduced
    on every rank.  Returns per-token latency and tokens/s for batch 1 and 32."""
    from qw6_b200 import synth as S
    from qw6_b200.lm_head import CudaLMHeadShard, shard_rows, sharded_argmax
    hbm, _ = peaks()
    V, H = S.VOCAB, HIDDEN
    r0, r1 = shard_rows(V, world, rank)
    rows = r1 - r0
    pb = ctx.packed_bytes(S.Q6_K, rows, H)
    w = torch.randint(0, 256, (pb,), dtype=torch.uint8, device="cuda")
    shard = CudaLMHeadShard(ctx, S.Q6_K, w.data_ptr(), rows, H, r0)
    res = {}
    for ntok in (1, 32):
        x = torch.randn((ntok, H), device="cuda")

        def one():
            with torch.cuda.stream(stream):
                sharded_argmax(shard, x, world)

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
    ctx.set_stream(stream.cuda_stream)
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


def c3_config():
    """config of the headline line (identical in both arms)."""
    return {"workload": "config 3: prefill MoE FFN layer, 4096 tokens", "tokens": T3, "hidden": HIDDEN,
            "experts": NE, "top_k": TOPK, "inter": INTER, "gate_up": "Q4_K", "down": "Q6_K",
            "router_bias": "N(0,0.5) per expert"}


def report(args, world, head, cpu):
    tflops_peak, tf_kind = bf16_peak()
    hbm, hbm_kind = peaks()
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
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16 (tcgen05 kind::f16, f32 accumulate; Q4_K/Q6_K weights)",
        "data": "synthetic (seeded GGUF blocks, config 3)",
        "config": c3_config(),
        "method": {"parallelism": f"ep{world}: {NE // world} experts and {T3 // world} tokens per GPU"
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
                "api": ("qw6cu_ep_layer_hostio" if world > 1 else "qw6cu_moe_prefill_hostio")
                       + " (one call over all steps)"
                       + ": every step copies this rank's logits/x in from pinned host memory and its fp32 output "
                         "back (per-rank bytes), pipelined over two device slots -- step s+1's copy-in and step "
                         "s-1's read-back run beside step s's experts; the timed region ends when the last "
                         "output is in host memory",
                "timing": (f"median of 3 timed calls of {head['e2e_steps']} steps each (ms per call: "
                           + ", ".join(f"{t:.2f}" for t in head["e2e_runs_ms"]) + ")"),
                "output_finite": head["finite"], "output_equals_device_steps": head["same"],
                "host_binding": (f"page-locked buffers from the NUMA node of the GPU's PCIe root ({head['host_cpus']} "
                                 "local CPUs)") if head["host_cpus"] else "unbound (no sysfs CPU list)"},
        "gpu_launches": int(launches * K),
        "clocks": head["clk"],
        "cpu_baseline": cpu,
    }


# --------------------------------------------------------- reference arm --

def decoder_step_bytes(model, pos: int) -> int:
    """Algorithmic HBM bytes of one decode step at position pos: every weight
    the step reads once (the 8 routed experts of each layer only), the fp32
    router, the DeltaNet states and conv windows read and written, the KV
    cache rows read (pos + 1 per attention layer) and the one written, the
    embedding row and the logits."""
    from qw6_b200 import synth as S
    n, seen = 0, set()
    for f, l, q, r, c, arr, stride in model.tensors:
        if f in (S.F_EXPERT_GATE, S.F_EXPERT_UP, S.F_EXPERT_DOWN):
            n += 8 * r * S.row_bytes(q, c)
        elif f == S.F_TOK_EMBD:
            n += S.row_bytes(q, c)
        else:
            n += r * S.row_bytes(q, c)
    for l in range(model.n_layers):
        if S.is_full_attn(l):
            n += (pos + 1) * 2 * 512 * 4 + 2 * 512 * 4
        else:
            n += 2 * (32 * 128 * 128 * 4 + 4 * 8192 * 4)
    return n + model.vocab * 4


def decoder_bench(args, ctx, L):
    """The decode-step executor on a full-size synthetic qw6 model (40 layers,
    distinct weights per layer: IQ2_XXS experts, Q6_K projections, shared
    expert, embeddings and LM head, 248320-token vocabulary): greedy tokens
    chained on the device (qw6cu_decoder_generate) and, end to end, one
    qw6cu_decoder_forward per token with the token id from the host and the
    pick (and optionally the logits) back.  Replicas only: a step is one
    token of one sequence; this runs on rank 0."""
    import torch
    from qw6_b200 import synth as S
    t0 = time.perf_counter()
    m = S.fwd_model(seed=31, n_layers=40, vocab=S.VOCAB, embd_rows=S.VOCAB, attn_period=40, expert_period=40)
    gen_s = time.perf_counter() - t0
    n = args.decoder_tokens
    dec = L.Decoder(ctx, m, max_ctx=max(4096, 2 * n + 64))
    dev_bytes = dec.device_bytes()
    step_bytes = [decoder_step_bytes(m, p) for p in range(n)]
    del m
    dec.generate(1, 0, 8)  # warm-up
    dec.reset()
    hbm, peak_kind = peaks()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    toks = dec.generate(1, 0, n)
    dt = time.perf_counter() - t0
    # end to end: host token in, pick back, every step synchronous
    dec.reset()
    tok, t1 = 1, time.perf_counter()
    for p in range(n):
        _, tok = dec.forward(tok, p, logits=False)
    e2e = time.perf_counter() - t1
    dec.reset()
    tok, t2 = 1, time.perf_counter()
    for p in range(min(n, 64)):
        _, tok = dec.forward(tok, p, logits=True)
    e2e_l = (time.perf_counter() - t2) / min(n, 64)
    dec.close()
    avg_bytes = sum(step_bytes) / n
    gbs = avg_bytes * n / dt / 1e9
    return {
        "workload": "decode-step executor: full qw6 forward pass per token (40 layers: 30 Gated DeltaNet + 10 gated "
                    "attention, MoE 256x top-8 IQ2_XXS + Q6_K shared expert, Q6_K projections / embeddings / LM head "
                    "248320) on one GPU, greedy, positions 0..n-1 (replicas only)",
        "data": "synthetic (seeded qw6 model, distinct weights per layer)",
        "tokens": n, "tokens_s": round(n / dt, 1), "ms_per_token": round(dt / n * 1e3, 4),
        "timing": "wall clock around qw6cu_decoder_generate (one CUDA graph replay per token, chained on the device, "
                  "one synchronization at the end)",
        "algorithmic_bytes_per_token": int(avg_bytes), "device_bytes": int(dev_bytes),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "peak_kind": peak_kind, "scope": "whole step"},
        "e2e": {"value": round(n / e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 16,
                "api": "qw6cu_decoder_forward per token (host token id in, greedy pick out, synchronous)",
                "with_logits_ms_per_token": round(e2e_l * 1e3, 4),
                "with_logits_d2h_bytes_per_step": S.VOCAB * 4 + 16},
        "first_tokens": [int(t) for t in toks[:8]],
        "model_generation_s": round(gen_s, 1),
    }


def run_reference(args, rank, world):
    """qw6's own CPU implementation of config 3's layer (oracle/_ref) on all
    usable host cores: each step runs a bounded sample of the 4096 tokens,
    sliced one token per task over a fork pool (qw6 is single-threaded).  The
    whole --steps/--warmup run is sized to end within a few minutes."""
    if rank != 0:
        return None
    from oracle.oracle import cpu_count
    from qw6_b200 import synth as S
    gate, up, down, lg, xb = S.config3()
    x = S.bf16_to_f32(xb)
    workers = cpu_count()
    one = CpuMoE(gate, up, down, lg, x, 1)
    one.run(1)
    t1 = one.run(2) / 2  # seconds per token on one core
    K, W = args.steps, args.warmup
    per_step_s = min(6.0, 150.0 / (K + W))
    per_step = workers * max(1, int(per_step_s / t1))
    pool = CpuMoE(gate, up, down, lg, x, workers)
    for _ in range(W):
        pool.run(per_step)
    dt = 0.0
    for _ in range(K):
        dt += pool.run(per_step)
    pool.close()
    value = K * per_step / dt
    return {
        "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(dt / K * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF blocks, config 3)",
        "config": c3_config(),
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": workers, "kind": "reference",
                         "sample": f"{per_step} of config 3's tokens per step (round robin over the 4096) on a fork "
                                   f"pool of {workers} processes, one token per task, each token through qw6's own "
                                   "qw6_cpu_moe_route and expert loop (qw6_tensor_matvec, qw6_silu; "
                                   "qw6.c:2246-2264) compiled from the reference sources (oracle/_ref); the "
                                   "reference has no batched path and is single-threaded, so the pool is the "
                                   "harness's; its Vulkan path is unavailable on this box",
                         "host": host_info()},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


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
    ap.add_argument("--no-decoder", dest="decoder", action="store_false",
                    help="skip the full-model decode-step executor leg")
    ap.add_argument("--decoder-tokens", type=int, default=256)
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
