"""Expert-parallel routed MoE for prefill batches.

The experts are sharded contiguously over the ranks of a process group
(rank r owns experts [r*E/G, (r+1)*E/G)); each rank holds its own tokens.
One layer (`ep_moe_prefill`):

  1. route this rank's tokens (top-k of their router logits);
  2. count the assignments of every global expert; one all-to-all gives each
     rank the counts of its own experts from every source;
  3. pack each assignment's bf16 token row into send rows sorted by global
     expert (so grouped by destination, and by local expert inside each
     destination's block);
  4. all-to-all the rows to their owners; the owner recovers each received
     row's expert from the exchanged counts;
  5. the owner runs the tensor-core grouped GEMMs over the rows it received
     (unweighted bf16 expert outputs);
  6. all-to-all the outputs back in send-row order;
  7. weight and sum each token's top-k outputs in slot order.

Steps 5-7 are the same arithmetic in the same order as the single-GPU
qw6cu_moe_prefill, so the result does not depend on the number of ranks.
Compute steps are libqw6cuda kernels (`CudaBackend`); the exchanges are
torch.distributed all-to-alls (NCCL between GPUs).  The orchestration is
backend-agnostic so that the same code runs on CPU gloo ranks in the tests.
Remote rows are always received into this rank's own memory before any
kernel reads them.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import lib as L

_CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: torch's default stream reports handle 0


class CudaBackend:
    """libqw6cuda kernels on the current rank's GPU (device tensors), issued
    on torch's current stream so they order with the collectives."""

    out_dtype = torch.bfloat16

    def __init__(self, ctx: L.Context, gate: L.ExpertPack, up: L.ExpertPack, down: L.ExpertPack, hidden: int,
                 inter: int, experts_per_rank: int):
        self.ctx, self.gate, self.up, self.down = ctx, gate, up, down
        self.hidden, self.inter, self.epr = hidden, inter, experts_per_rank
        self.device = torch.device("cuda", torch.cuda.current_device())

    def _bind(self):
        self.ctx.set_stream(torch.cuda.current_stream(self.device).cuda_stream or _CUDA_STREAM_LEGACY)
        return self.ctx

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype, device=self.device)

    def route(self, logits, ntok, n_experts, top_k):
        idx = self.empty((ntok * top_k,), torch.int32)
        w = self.empty((ntok * top_k,), torch.float32)
        self._bind().moe_route(logits.data_ptr(), ntok, n_experts, top_k, idx.data_ptr(), w.data_ptr())
        return idx, w

    def place(self, idx, eslot):
        """Routed expert ids -> placed ids (eslot: int32 numpy [n_experts])."""
        return torch.as_tensor(eslot, device=self.device).index_select(0, idx.long()).to(torch.int32)

    def count(self, idx, n, n_experts):
        cnt = self.empty((n_experts,), torch.int32)
        pos = self.empty((n,), torch.int32)
        self._bind().ep_count(idx.data_ptr(), n, n_experts, cnt.data_ptr(), pos.data_ptr())
        return cnt, pos

    def pack(self, idx, pos, cnt, n, top_k, n_experts, x):
        send_x = self.empty((n, self.hidden), torch.bfloat16)
        send_pos = self.empty((n,), torch.int32)
        self._bind().ep_pack(idx.data_ptr(), pos.data_ptr(), cnt.data_ptr(), n, top_k, n_experts, x.data_ptr(),
                             self.hidden, send_x.data_ptr(), send_pos.data_ptr())
        return send_x, send_pos

    def expand(self, recv_cnt, world, nrecv):
        row_e = self.empty((max(nrecv, 1),), torch.int32)
        self._bind().ep_expand(recv_cnt.data_ptr(), world, self.epr, row_e.data_ptr())
        return row_e

    def expert_rows(self, recv_x, row_e, nrecv):
        out = self.empty((nrecv, self.hidden), torch.bfloat16)
        if nrecv:
            self._bind().moe_expert_rows(self.gate, self.up, self.down, recv_x.data_ptr(), row_e.data_ptr(),
                                         out.data_ptr(), nrecv, self.hidden, self.inter, self.epr)
        return out

    def combine(self, ret, w, send_pos, ntok, top_k):
        out = self.empty((ntok, self.hidden), torch.float32)
        self._bind().ep_combine(ret.data_ptr(), w.data_ptr(), send_pos.data_ptr(), ntok, top_k, self.hidden,
                                out.data_ptr())
        return out

    def local_layer(self, logits, x, ntok, n_experts, top_k):
        """All experts on this GPU: the single-GPU qw6cu_moe_prefill."""
        out = self.empty((ntok, self.hidden), torch.float32)
        self._bind().moe_prefill(self.gate, self.up, self.down, logits.data_ptr(), x.data_ptr(), out.data_ptr(), ntok,
                                 self.hidden, self.inter, n_experts, top_k)
        return out


def placement_slots(placement, world: int, n_experts: int):
    """Validate an expert placement ([world, n_experts/world] routed ids, as
    from `balance_experts`) and return (eslot, identity): eslot[routed id] =
    placed id (rank * epr + local index) as int32."""
    pl = np.asarray(placement, dtype=np.int64)
    if pl.shape != (world, n_experts // world):
        raise ValueError(f"placement must have shape ({world}, {n_experts // world})")
    flat = pl.reshape(-1)
    if not np.array_equal(np.sort(flat), np.arange(n_experts)):
        raise ValueError("placement is not a permutation of the experts")
    eslot = np.empty(n_experts, np.int32)
    eslot[flat] = np.arange(n_experts, dtype=np.int32)
    return eslot, bool(np.array_equal(flat, np.arange(n_experts)))


def _all_to_all(out, inp, out_splits=None, in_splits=None, group=None):
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        out.copy_(inp)
    else:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


def ep_moe_prefill(backend, logits: torch.Tensor, x_bf16: torch.Tensor, top_k: int, n_experts: int,
                   group=None, stats: dict | None = None, placement=None) -> torch.Tensor:
    """One routed-MoE layer for this rank's tokens with experts sharded over
    `group`.  logits [T x n_experts] fp32, x_bf16 [T x hidden] bf16 (this
    rank's tokens); returns out [T x hidden] fp32.  Without a process group
    (or with one rank) the backend holds all experts and runs the layer
    locally.  `placement` (None: rank r holds experts [r*epr, (r+1)*epr)) is
    an int array [world, epr] as from `balance_experts`, the same on every
    rank; the backend's local expert j is then placement[rank][j].  Results
    do not depend on it.  `stats`, when given, receives the number of rows
    this rank's experts processed ("rows")."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    ntok, hidden = x_bf16.shape
    n = ntok * top_k
    if n_experts % world or n_experts > 256:
        raise ValueError(f"{n_experts} experts do not shard evenly over {world} ranks")
    eslot, identity = placement_slots(placement, world, n_experts) if placement is not None else (None, True)
    if world == 1 and identity and hasattr(backend, "local_layer"):
        if stats is not None:
            stats["rows"] = n
        return backend.local_layer(logits, x_bf16, ntok, n_experts, top_k)
    epr = n_experts // world
    idx, w = backend.route(logits, ntok, n_experts, top_k)
    if not identity:  # every later step works in placed ids: owner = id // epr
        idx = backend.place(idx, eslot)
    cnt, pos = backend.count(idx, n, n_experts)
    recv_cnt = torch.empty_like(cnt)  # [source][local expert]
    _all_to_all(recv_cnt, cnt, group=group)
    counts = torch.cat([cnt, recv_cnt]).cpu()  # split sizes are host-side lists
    send_counts = counts[:n_experts].view(world, epr).sum(1).tolist()
    recv_counts = counts[n_experts:].view(world, epr).sum(1).tolist()
    nrecv = sum(recv_counts)
    if stats is not None:
        stats["rows"] = nrecv
    send_x, send_pos = backend.pack(idx, pos, cnt, n, top_k, n_experts, x_bf16)
    recv_x = backend.empty((nrecv, hidden), x_bf16.dtype)
    _all_to_all(recv_x, send_x, recv_counts, send_counts, group=group)
    row_e = backend.expand(recv_cnt, world, nrecv)
    recv_out = backend.expert_rows(recv_x, row_e, nrecv)
    ret = backend.empty((n, hidden), recv_out.dtype)
    _all_to_all(ret, recv_out, send_counts, recv_counts, group=group)
    return backend.combine(ret, w, send_pos, ntok, top_k)


def balance_experts(counts, world: int) -> "np.ndarray":
    """Expert placement for `world` ranks from per-expert routing counts
    (rows per expert over a calibration sample), the same idea as an
    expert-parallel load balancer: every rank holds n_experts/world experts
    and the ranks' row totals are evened out -- experts in decreasing count
    go to the least-loaded rank with room left, then pairs are swapped
    between the heaviest rank and a lighter one while that lowers the
    heavier total.  Returns int32 [world, n_experts/world] (rank r's experts,
    ascending); flattened it is the `experts` array of qw6cu_ep_set_placement.
    Placement never changes a result bit: each expert's rows go through the
    same GEMM arithmetic on whichever rank holds it."""
    counts = np.asarray(counts, dtype=np.int64)
    ne = counts.shape[0]
    if world < 1 or ne % world:
        raise ValueError("n_experts must be a multiple of world")
    epr = ne // world
    members = [[] for _ in range(world)]
    load = np.zeros(world, np.int64)
    for g in np.argsort(-counts, kind="stable"):
        r = min((r for r in range(world) if len(members[r]) < epr), key=lambda r: (load[r], r))
        members[r].append(int(g))
        load[r] += counts[g]
    while True:  # every swap lowers the sum of squared loads, so this ends
        hi = int(np.argmax(load))
        done = True
        for lo in np.argsort(load, kind="stable"):
            gap = load[hi] - load[lo]
            if lo == hi or gap <= 1:
                continue
            ca = counts[members[hi]][:, None]
            cb = counts[members[lo]][None, :]
            d = ca - cb
            score = np.where((d > 0) & (d < gap), np.abs(gap - 2 * d), np.iinfo(np.int64).max)
            i, j = np.unravel_index(int(np.argmin(score)), score.shape)
            if score[i, j] == np.iinfo(np.int64).max:
                continue
            a, b = members[hi][i], members[lo][j]
            members[hi][i], members[lo][j] = b, a
            load[hi] -= counts[a] - counts[b]
            load[lo] += counts[a] - counts[b]
            done = False
            break
        if done:
            return np.array([sorted(m) for m in members], dtype=np.int32)


class PeerMoE:
    """The peer-memory expert-parallel layer (libqw6cuda qw6cu_ep_*): token
    rows and expert outputs move over NVLink by loads/stores in this
    library's own kernels, with no host synchronisation inside a layer, so a
    step can be captured in a CUDA graph.  Construction is collective over
    `group`: every rank allocates its symmetric region and the CUDA IPC
    handles are all-gathered.  Results are bit-identical to
    `ep_moe_prefill` and to the single-GPU layer."""

    def __init__(self, ctx: L.Context, gate: L.ExpertPack, up: L.ExpertPack, down: L.ExpertPack, n_experts: int,
                 top_k: int, hidden: int, inter: int, max_tokens: int, group=None, placement=None):
        """placement: None (rank r holds experts [r*epr, (r+1)*epr)) or an
        int array [world, epr] as from `balance_experts`, the same on every
        rank; the packs then hold this rank's row of it, in that order."""
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.ctx, self.packs, self.hidden, self.max_tokens = ctx, (gate, up, down), hidden, max_tokens
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.ep = L.PeerEP(ctx, rank, world, n_experts, top_k, hidden, inter, max_tokens)
        mine = self.ep.handle()
        if world > 1:
            allh = [None] * world
            dist.all_gather_object(allh, mine, group=group)
        else:
            allh = [mine]
        self.ep.connect(allh)
        if placement is not None:
            placement_slots(placement, world, n_experts)  # shape and permutation checks
            self.ep.set_placement(np.asarray(placement, dtype=np.int64).reshape(-1))
        if world > 1:
            dist.barrier(group=group)

    def __call__(self, logits: torch.Tensor, x_bf16: torch.Tensor, out: torch.Tensor | None = None,
                 packs: tuple | None = None) -> torch.Tensor:
        """One layer step on torch's current stream (`packs` overrides the
        expert packs given at construction, e.g. another layer's)."""
        ntok = x_bf16.shape[0]
        if out is None:
            out = torch.empty((ntok, self.hidden), dtype=torch.float32, device=self.device)
        self.ctx.set_stream(torch.cuda.current_stream(self.device).cuda_stream or _CUDA_STREAM_LEGACY)
        self.ep.layer(*(packs or self.packs), logits.data_ptr(), x_bf16.data_ptr(), out.data_ptr(), ntok)
        return out

    def hostio(self, logits_host, x_host, out_host, ntok: int, packs: tuple | None = None) -> None:
        """Layer steps whose inputs and outputs are in host memory (one host
        address per step in each sequence; qw6cu_ep_layer_hostio): copies
        pipelined with the steps on the context's stream, synchronous."""
        self.ctx.set_stream(torch.cuda.current_stream(self.device).cuda_stream or _CUDA_STREAM_LEGACY)
        self.ep.layer_hostio(*(packs or self.packs), logits_host, x_host, out_host, ntok)

    def last_rows(self) -> int:
        return self.ep.last_rows()

    def close(self):
        self.ep.close()

