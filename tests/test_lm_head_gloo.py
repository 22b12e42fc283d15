"""CPU: the row-sharded LM head (qw6_b200/lm_head.py) on 2 and 3 gloo ranks.

Each rank holds its `shard_rows` slice of a Q6_K output projection; a CPU
backend computes the shard's logits with the oracle (qw6's matvec) and packs
them into (logit, global row) keys the way qw6cu_lm_head_argmax does; the
partition, the all-gather and the reduction order are the production code.
The token must equal the oracle's qw6_cpu_argmax over the full logits,
including a tie planted across the shard boundary (lowest row wins) and a NaN
at row 0 (qw6's scan never moves past it)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qw6_b200 import synth as S

V, H, NTOK = 1000, 512, 3


def pack_key(v: np.float32, i: int) -> int:
    """qw6_argmax.cuh argmax_key: ordered(value) << 32 | ~index."""
    if np.isnan(v):
        if i == 0:
            return -1  # all ones as int64
        u = 0x007FFFFF
    else:
        b = int(np.float32(v).view(np.uint32))
        u = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    k = (u << 32) | (~i & 0xFFFFFFFF)
    return k - (1 << 64) if k >= 1 << 63 else k


def unpack_key(k: int):
    k &= (1 << 64) - 1
    if k == (1 << 64) - 1:
        return 0, float("nan")
    u, i = k >> 32, ~k & 0xFFFFFFFF
    b = (u & 0x7FFFFFFF) if u & 0x80000000 else (~u & 0xFFFFFFFF)
    return i, float(np.uint32(b).view(np.float32))


class OracleShard:
    def __init__(self, w_rows, r0, rows):
        from oracle.oracle import Oracle
        self.o, self.w, self.r0, self.rows = Oracle(), w_rows, r0, rows

    def keys(self, x, keys):
        for t in range(x.shape[0]):
            lg = self.o.matvec(S.Q6_K, self.w, x[t].numpy(), self.rows, H)
            best = None
            for r in range(self.rows):
                k = pack_key(lg[r], self.r0 + r)
                if best is None or (k & ((1 << 64) - 1)) > (best & ((1 << 64) - 1)):
                    best = k
            keys[t] = best

    def reduce(self, allk, nshards, ntok, idx, val):
        a = allk.numpy().reshape(nshards, ntok)
        for t in range(ntok):
            k = max((int(a[s, t]) & ((1 << 64) - 1) for s in range(nshards)))
            i, v = unpack_key(k)
            idx[t], val[t] = i, v


def _data(case):
    rng = np.random.Generator(np.random.PCG64(41))
    w = S.make_matrix(S.Q6_K, V, H, rng)
    x = rng.standard_normal((NTOK, H), dtype=np.float32)
    if case == "tie":  # rows 12 and 990 identical: equal logits on different shards
        from oracle.oracle import Oracle
        w[990] = w[12]
        # token 1 points along row 12, so the two equal logits are the largest
        x[1] = Oracle().dequantize(S.Q6_K, w[12:13], 1, H)[0]
    if case == "nan0":
        w[0, 208:210] = np.array([0x00, 0x7E], np.uint8)  # d of row 0's first block: fp16 NaN
    return w, x


def _rank(rank, world, port, case, q):
    from qw6_b200.lm_head import shard_rows, sharded_argmax
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, x = _data(case)
        r0, r1 = shard_rows(V, world, rank)
        be = OracleShard(np.ascontiguousarray(w[r0:r1]), r0, r1 - r0)
        idx, val = sharded_argmax(be, torch.from_numpy(x), world)
        q.put((rank, idx.numpy().copy(), val.numpy().copy(), (r0, r1)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case", ["random", "tie", "nan0"])
@pytest.mark.parametrize("world", [2, 3])
def test_sharded_lm_head_gloo(world, case, oracle):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort(key=lambda g: g[0])
    spans = [g[3] for g in got]
    assert spans[0][0] == 0 and spans[-1][1] == V and all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
    w, x = _data(case)
    full = oracle.matvec(S.Q6_K, w, x, V, H).reshape(NTOK, V)
    for r in range(world):  # every rank holds the same answer
        assert np.array_equal(got[r][1], got[0][1])
    for t in range(NTOK):
        want = oracle.argmax(full[t])
        assert got[0][1][t] == want, (t, got[0][1][t], want)
        if not np.isnan(full[t][want]):
            assert got[0][2][t] == full[t][want]
    if case == "tie":  # the two maximal logits are equal; the lower row wins across the shard boundary
        assert full[1][12] == full[1][990] == np.max(full[1])
        assert got[0][1][1] == 12
