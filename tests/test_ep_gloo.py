"""CPU: the expert-parallel orchestration (qw6_b200/ep.py) on 2 gloo ranks.

The compute steps run through a numpy backend built on the CPU oracle; the
dispatch/combine bookkeeping, the split sizes and the all-to-all sequence are
the production code.  The result must equal the oracle's single-process
routed MoE on the same tokens (the oracle's expert FFN is fp32 on the
bf16-widened rows, as qw6_apply_layer_moe composes it)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qw6_b200 import synth as S

E, H, I, K, T_PER_RANK = 8, 512, 512, 4, 24


class OracleBackend:
    """ep.py backend contract, implemented on the CPU with the oracle
    (fp32 expert outputs instead of the GPU's bf16)."""

    out_dtype = torch.float32

    def __init__(self, gate, up, down, epr, rank, experts=None):
        from oracle.oracle import Oracle
        self.o = Oracle()
        self.gate, self.up, self.down, self.epr, self.rank = gate, up, down, epr, rank
        # routed id of local expert j (contiguous sharding unless placed)
        self.experts = list(range(rank * epr, (rank + 1) * epr)) if experts is None else [int(e) for e in experts]

    def place(self, idx, eslot):
        return torch.from_numpy(np.asarray(eslot)[idx.numpy()].astype(np.int32))

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype)

    def route(self, logits, ntok, n_experts, top_k):
        idx, w = zip(*(self.o.moe_route(logits[t].numpy(), top_k) for t in range(ntok)))
        return torch.from_numpy(np.concatenate(idx)), torch.from_numpy(np.concatenate(w))

    def count(self, idx, n, n_experts):
        e = idx.numpy()
        cnt = np.bincount(e, minlength=n_experts).astype(np.int32)
        pos = np.zeros(n, np.int32)
        seen = np.zeros(n_experts, np.int32)
        for a in range(n - 1, -1, -1):  # any order is valid; reverse assignment order
            pos[a] = seen[e[a]]
            seen[e[a]] += 1
        return torch.from_numpy(cnt), torch.from_numpy(pos)

    def pack(self, idx, pos, cnt, n, top_k, n_experts, x):
        off = np.concatenate([[0], np.cumsum(cnt.numpy())[:-1]])
        p = off[idx.numpy()] + pos.numpy()
        send_x = torch.empty((n, x.shape[1]), dtype=x.dtype)
        send_x[torch.from_numpy(p).long()] = x[torch.arange(n) // top_k]
        return send_x, torch.from_numpy(p.astype(np.int32))

    def expand(self, recv_cnt, world, nrecv):
        e = np.tile(np.arange(self.epr, dtype=np.int32), world)
        return torch.from_numpy(np.repeat(e, recv_cnt.numpy()))

    def expert_rows(self, recv_x, row_e, nrecv):
        out = np.zeros((nrecv, H), np.float32)
        xs = recv_x.float().numpy()
        for r in range(nrecv):
            e = self.experts[int(row_e[r])]
            g = self.o.matvec(S.Q4_K, self.gate[e], xs[r], I, H)
            u = self.o.matvec(S.Q4_K, self.up[e], xs[r], I, H)
            out[r] = self.o.matvec(S.Q6_K, self.down[e], self.o.silu_mul(g, u), H, I)
        return torch.from_numpy(out)

    def combine(self, ret, w, send_pos, ntok, top_k):
        r = ret.numpy()
        sp = send_pos.numpy().reshape(ntok, top_k)
        ww = w.numpy().reshape(ntok, top_k)
        out = np.zeros((ntok, H), np.float32)
        for k in range(top_k):
            out += ww[:, k:k + 1] * r[sp[:, k]]
        return torch.from_numpy(out)


def _data():
    rng = np.random.Generator(np.random.PCG64(808))
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((2 * T_PER_RANK, E), dtype=np.float32)
    xbits = S.bf16_round(rng.standard_normal((2 * T_PER_RANK, H), dtype=np.float32))
    return gate, up, down, logits, xbits


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qw6_b200.ep import ep_moe_prefill
        gate, up, down, logits, xbits = _data()
        sl = slice(rank * T_PER_RANK, (rank + 1) * T_PER_RANK)
        x = torch.from_numpy(S.bf16_to_f32(xbits[sl])).to(torch.bfloat16)
        be = OracleBackend(gate, up, down, E // world, rank)
        out = ep_moe_prefill(be, torch.from_numpy(logits[sl]), x, K, E)
        # the same layer with the experts placed by a permutation
        pl = np.random.Generator(np.random.PCG64(41)).permutation(E).reshape(world, E // world)
        bp = OracleBackend(gate, up, down, E // world, rank, experts=pl[rank])
        stats = {}
        outp = ep_moe_prefill(bp, torch.from_numpy(logits[sl]), x, K, E, stats=stats, placement=pl)
        q.put((rank, (out.numpy(), outp.numpy(), stats["rows"])))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_prefill_two_gloo_ranks(oracle):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gate, up, down, logits, xbits = _data()
    ref, _, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, S.bf16_to_f32(xbits), top_k=K)
    out = np.concatenate([got[0][0], got[1][0]])
    err = float(np.max(np.abs(out - ref)) / np.max(np.abs(ref)))
    assert err <= 1e-5, err
    # placement changes which rank computes an expert, never a result bit
    outp = np.concatenate([got[0][1], got[1][1]])
    assert np.array_equal(outp.view(np.uint32), out.view(np.uint32))
    assert got[0][2] + got[1][2] == 2 * T_PER_RANK * K


def test_placement_slots():
    from qw6_b200.ep import placement_slots
    eslot, ident = placement_slots([[2, 0], [3, 1]], 2, 4)
    assert eslot.tolist() == [1, 3, 0, 2] and not ident
    assert placement_slots(np.arange(4).reshape(2, 2), 2, 4)[1]
    with pytest.raises(ValueError):
        placement_slots([[0, 0], [1, 2]], 2, 4)  # not a permutation
    with pytest.raises(ValueError):
        placement_slots([[0, 1, 2, 3]], 2, 4)  # wrong shape


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_balance_experts(world):
    """Placement: a permutation with n_experts/world experts per rank, no
    heavier than contiguous sharding, within one expert's count of the mean
    on config 3's skewed routing, and the same on every call."""
    from qw6_b200.ep import balance_experts
    _, _, _, logits, _, bias = S.config3(ntok=1024, with_bias=True)
    cnt = np.bincount(np.argsort(-logits, axis=1, kind="stable")[:, :8].ravel(), minlength=logits.shape[1])
    pl = balance_experts(cnt, world)
    ne = cnt.shape[0]
    assert pl.shape == (world, ne // world)
    assert np.array_equal(np.sort(pl.reshape(-1)), np.arange(ne))
    load = cnt[pl].sum(axis=1)
    contiguous = cnt.reshape(world, -1).sum(axis=1)
    assert load.max() <= contiguous.max()
    assert load.max() - cnt.sum() / world <= cnt.max(), (load, cnt.max())
    assert np.array_equal(pl, balance_experts(cnt, world))
    # an independent batch of the same router balances the measured one almost as well
    cal = S.router_sample(bias, 1024, seed=11)
    ccnt = np.bincount(np.argsort(-cal, axis=1, kind="stable")[:, :8].ravel(), minlength=ne)
    if world > 1:
        assert cnt[balance_experts(ccnt, world)].sum(axis=1).max() < contiguous.max()


def test_balance_experts_edges():
    from qw6_b200.ep import balance_experts
    assert np.array_equal(balance_experts(np.zeros(8, np.int64), 2), [[0, 1, 2, 3], [4, 5, 6, 7]])  # ties: contiguous
    pl = balance_experts([100, 0, 0, 0], 4)
    assert sorted(pl.reshape(-1).tolist()) == [0, 1, 2, 3]
    with pytest.raises(ValueError):
        balance_experts(np.ones(6), 4)
