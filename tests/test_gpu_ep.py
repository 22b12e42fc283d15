"""GPU: expert-parallel prefill MoE, NCCL and peer-memory variants.

Each of `world` ranks (one spawned process per GPU) owns E/world experts and
T/world tokens and runs (a) qw6_b200.ep.ep_moe_prefill over NCCL
all-to-alls and (b) qw6_b200.ep.PeerMoE (libqw6cuda's own dispatch/combine
kernels over peer memory) three times in a row and once more as a replayed
CUDA graph; then both with the experts placed by a permutation.  Every
gathered output must equal, bit for bit, the single-GPU
qw6cu_moe_prefill on all tokens (same expert outputs, same slot-order
combine), and match the oracle's expert-grouped float64 recomputation on every
token and its fp32 composition on a seeded sample of tokens within 2e-2 (the
bf16 tensor-core prefill tolerance).  world=1 runs
on any GPU box; larger worlds are skipped when the box has fewer GPUs."""
import os
import socket

import numpy as np
import pytest

from qw6_b200 import synth as S

pytestmark = pytest.mark.gpu

E, H, I, K, T = 32, 2048, 512, 8, 512


def _data(case):
    rng = np.random.Generator(np.random.PCG64(909))
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    bias = (rng.standard_normal(E) * 0.5).astype(np.float32)
    logits = (rng.standard_normal((T, E), dtype=np.float32) + bias).astype(np.float32)
    if case == "upper_half_idle":  # no token routes to experts E/2.. (their owners receive nothing)
        logits[:, E // 2:] = -1e4
    xbits = S.bf16_round(rng.standard_normal((T, H), dtype=np.float32))
    return gate, up, down, logits, xbits


def _pack_all(ctx, torch, L, mats, lo, hi, ids=None):
    packs, held = [], []
    ids = np.arange(lo, hi) if ids is None else np.asarray(ids)
    for qq, m, r, c in mats:
        mine = np.ascontiguousarray(m[ids])
        pb = ctx.packed_bytes(qq, r, c)
        raw = torch.from_numpy(mine.reshape(-1)).cuda()
        pk = torch.empty(pb * len(ids), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ctx.pack(qq, raw.data_ptr(), pk.data_ptr(), r, c, len(ids), mine[0].nbytes, pb)
        ctx.synchronize()
        held.append(pk)
        packs.append(L.ExpertPack(qq, pk.data_ptr(), pb))
    return packs, held


def _rank(rank, world, port, case, q):
    import torch
    import torch.distributed as dist

    from qw6_b200 import lib as L
    from qw6_b200.ep import CudaBackend, PeerMoE, ep_moe_prefill

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        gate, up, down, logits, xbits = _data(case)
        mats = ((S.Q4_K, gate, I, H), (S.Q4_K, up, I, H), (S.Q6_K, down, H, I))
        epr, tpr = E // world, T // world
        ctx = L.Context(rank)
        packs, held = _pack_all(ctx, torch, L, mats, rank * epr, (rank + 1) * epr)
        be = CudaBackend(ctx, packs[0], packs[1], packs[2], H, I, epr)
        sl = slice(rank * tpr, (rank + 1) * tpr)
        lg = torch.from_numpy(logits[sl]).cuda()
        x = torch.from_numpy(xbits[sl].view(np.int16)).cuda().view(torch.bfloat16)
        torch.cuda.synchronize()
        out = ep_moe_prefill(be, lg, x, K, E)
        torch.cuda.synchronize()
        ctx.check_device_errors()
        # peer-memory layer: repeated steps reuse the buffers (epochs 1..3) ...
        pm = PeerMoE(ctx, packs[0], packs[1], packs[2], E, K, H, I, tpr)
        peer = [pm(lg, x).cpu().numpy() for _ in range(3)]
        ctx.check_device_errors()
        # ... and a captured step replays with fresh epochs
        s = torch.cuda.Stream()
        gout = torch.empty((tpr, H), dtype=torch.float32, device="cuda")
        gout.fill_(float("nan"))
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            pm(lg, x, gout)
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        ctx.check_device_errors()
        peer.append(gout.cpu().numpy())
        del g
        # ... and steps whose inputs and outputs are in host memory, pipelined
        # over the two device slots (qw6cu_ep_layer_hostio)
        hl = torch.from_numpy(logits[sl]).pin_memory()
        hx = torch.from_numpy(xbits[sl].view(np.int16)).pin_memory()
        ho = [torch.full((tpr, H), float("nan")).pin_memory() for _ in range(3)]
        torch.cuda.synchronize()
        pm.hostio([hl.data_ptr()] * 3, [hx.data_ptr()] * 3, [o.data_ptr() for o in ho], tpr)
        ctx.check_device_errors()
        peer += [ho[0].numpy().copy(), ho[2].numpy().copy()]
        pm.close()
        # experts placed by a (seeded) permutation instead of contiguous blocks
        pl = np.random.Generator(np.random.PCG64(77)).permutation(E).reshape(world, epr).astype(np.int32)
        ppacks, pheld = _pack_all(ctx, torch, L, mats, 0, 0, pl[rank])
        pm = PeerMoE(ctx, ppacks[0], ppacks[1], ppacks[2], E, K, H, I, tpr, placement=pl)
        peer.append(pm(lg, x).cpu().numpy())
        ctx.check_device_errors()
        pm.close()
        # ... and the NCCL form with the same placement
        ctx.set_stream(None)
        bp = CudaBackend(ctx, ppacks[0], ppacks[1], ppacks[2], H, I, epr)
        torch.cuda.synchronize()
        peer.append(ep_moe_prefill(bp, lg, x, K, E, placement=pl).cpu().numpy())
        ctx.check_device_errors()
        del pheld
        full = None
        if rank == 0:  # single-GPU reference over all tokens and experts
            ctx.set_stream(None)
            fpacks, fheld = _pack_all(ctx, torch, L, mats, 0, E)
            lga = torch.from_numpy(logits).cuda()
            xa = torch.from_numpy(xbits.view(np.int16)).cuda()
            fo = torch.empty((T, H), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            ctx.moe_prefill(fpacks[0], fpacks[1], fpacks[2], lga.data_ptr(), xa.data_ptr(), fo.data_ptr(), T, H, I,
                            E, K)
            ctx.synchronize()
            ctx.check_device_errors()
            full = fo.cpu().numpy()
        q.put((rank, out.cpu().numpy(), peer, full))
        ctx.close()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case", ["spread", "upper_half_idle"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ep_prefill_nccl(world, case, oracle):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, o, pr, f = q.get(timeout=600)
        got[r] = (o, pr, f)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    out = np.concatenate([got[r][0] for r in range(world)])
    full = got[0][2]
    assert np.array_equal(out.view(np.uint32), full.view(np.uint32)), float(np.max(np.abs(out - full)))
    for i in range(8):  # three eager peer steps, the graph replay, two host-buffer steps, the permuted placement
        # (peer, NCCL)
        peer = np.concatenate([got[r][1][i] for r in range(world)])
        assert np.array_equal(peer.view(np.uint32), full.view(np.uint32)), (i, float(np.nanmax(np.abs(peer - full))))
    gate, up, down, logits, xbits = _data(case)
    # every token against the expert-grouped float64 recomputation ...
    ref64, _, _ = oracle.moe_layer_grouped_f64(S.Q4_K, gate, up, S.Q6_K, down, logits, S.bf16_to_f32(xbits),
                                               top_k=K)
    errs = [float(np.max(np.abs(out[t] - ref64[t])) / np.max(np.abs(ref64[t]))) for t in range(T)]
    assert max(errs) <= 2e-2, max(errs)
    # ... and a seeded sample against the fp32 oracle (qw6's evaluation order)
    toks = np.random.Generator(np.random.PCG64(5)).choice(T, 64, replace=False)
    ref, _, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits[toks], S.bf16_to_f32(xbits[toks]), top_k=K)
    errs = [float(np.max(np.abs(out[t] - ref[i])) / np.max(np.abs(ref[i]))) for i, t in enumerate(toks)]
    assert max(errs) <= 2e-2, max(errs)


def _rank_skip(rank, world, port, q):
    """Rank 1 takes part in one step, then skips the next; rank 0 runs it
    with a 300 ms limit on its cross-GPU waits."""
    import datetime
    import re
    import time

    import torch
    import torch.distributed as dist

    from qw6_b200 import lib as L
    from qw6_b200.ep import PeerMoE

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        gate, up, down, logits, xbits = _data("spread")
        mats = ((S.Q4_K, gate, I, H), (S.Q4_K, up, I, H), (S.Q6_K, down, H, I))
        epr, tpr = E // world, T // world
        ctx = L.Context(rank)
        packs, held = _pack_all(ctx, torch, L, mats, rank * epr, (rank + 1) * epr)
        sl = slice(rank * tpr, (rank + 1) * tpr)
        lg = torch.from_numpy(logits[sl]).cuda()
        x = torch.from_numpy(xbits[sl].view(np.int16)).cuda().view(torch.bfloat16)
        pm = PeerMoE(ctx, packs[0], packs[1], packs[2], E, K, H, I, tpr)
        pm(lg, x)  # a complete step on both ranks
        torch.cuda.synchronize()
        ctx.check_device_errors()
        pm.ep.set_wait_limit(300)
        dist.barrier()
        code, dt = 0, 0.0
        if rank == 0:  # rank 1 launches nothing for this step
            t0 = time.perf_counter()
            pm(lg, x)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            try:
                ctx.check_device_errors()
            except L.Qw6CudaError as e:
                m = re.search(r"code (\d+)", str(e))
                code = int(m.group(1)) if m else -1
        dist.barrier()
        pm.close()
        del held
        q.put((rank, code, dt))
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_ep_peer_rank_skips_a_step():
    """Failure detection without a GPU fault: when a peer stops taking part
    between steps, the other rank's bounded waits give up after the
    endpoint's limit, the context reports a timeout with the wait's kind
    (error word 41-44), the layer's later phases do nothing, and both
    processes exit normally."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_skip, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, code, dt = q.get(timeout=300)
        got[r] = (code, dt)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    code, dt = got[0]
    assert 41 <= code <= 44, code
    assert dt < 5.0, dt
    assert got[1][0] == 0
