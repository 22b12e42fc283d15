"""Row-sharded LM head with greedy argmax over N ranks (one process per GPU).

qw6 computes the logits of the whole vocabulary and scans them with
qw6_cpu_argmax (qw6.c:2493, 2858-2863).  Here rank r holds the rows
[r0, r1) of the output projection (`shard_rows`, rounded to 16-row tiles)
and reduces its shard to one packed (logit, row) key per token
(qw6cu_lm_head_argmax: larger logit first, lower global row on ties, NaN at
row 0 wins as in the CPU scan); the ranks all-gather their 8-byte keys and
take the maximum (qw6cu_argmax_keys_reduce).  The maximum of keys is
associative, so the token equals qw6's scan of the full logits whatever the
number of shards.

The compute steps go through a backend (`CudaLMHeadShard` on a GPU); the
partition and the collective are this module's, so a CPU backend can drive
the same code on gloo ranks.
"""
from __future__ import annotations

import torch

from . import lib as L


def shard_rows(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of the vocabulary that `rank` of `world` holds: equal
    shares rounded down to 16-row tiles, the last rank takes the rest."""
    r0 = (vocab * rank // world) // 16 * 16
    r1 = vocab if rank == world - 1 else (vocab * (rank + 1) // world) // 16 * 16
    return r0, r1


class CudaLMHeadShard:
    """Backend on this rank's GPU: the shard's packed rows in device memory."""

    def __init__(self, ctx: L.Context, quant: int, packed_ptr: int, rows: int, cols: int, row_offset: int):
        self.ctx, self.quant, self.w, self.rows, self.cols, self.r0 = ctx, quant, packed_ptr, rows, cols, row_offset

    def keys(self, x: torch.Tensor, keys: torch.Tensor) -> None:
        """keys[t] (int64, device) = this shard's packed max of token t."""
        self.ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        self.ctx.lm_head_argmax(self.quant, self.w, x.data_ptr(), x.shape[0], self.rows, self.cols, self.r0,
                                keys.data_ptr())

    def reduce(self, allk: torch.Tensor, nshards: int, ntok: int, idx: torch.Tensor, val: torch.Tensor) -> None:
        self.ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        self.ctx.argmax_keys_reduce(allk.data_ptr(), nshards, ntok, idx.data_ptr(), val.data_ptr())


def sharded_argmax(backend, x: torch.Tensor, world: int, group=None):
    """Greedy token of every row of x over the sharded vocabulary: this
    shard's keys, an all-gather of the world's keys (8 bytes per token and
    rank), the exact key reduction.  Returns (idx int32 [ntok], logit fp32
    [ntok]) on every rank."""
    ntok = x.shape[0]
    keys = torch.zeros(ntok, dtype=torch.int64, device=x.device)
    backend.keys(x, keys)
    if world > 1:
        import torch.distributed as dist
        allk = torch.empty(world * ntok, dtype=torch.int64, device=x.device)
        dist.all_gather_into_tensor(allk, keys, group=group)
    else:
        allk = keys
    idx = torch.empty(ntok, dtype=torch.int32, device=x.device)
    val = torch.empty(ntok, dtype=torch.float32, device=x.device)
    backend.reduce(allk, world, ntok, idx, val)
    return idx, val
