"""GPU sampling (qw6cu_sample) against qw6_sample (qw6.c:2904-2982): the
golden fixture of qw6's own picks (21 draws over full 248320-entry rows with
tied maxima) and the oracle on rows built to stress the order rule (many
tied scores, so the lower index must win inside a tie) and each branch
(greedy, top-k, top-p, plain temperature, top-k of 1).  A pick may differ
from the CPU only when u * sum lies within rounding of a cumulative boundary;
the draws here are far from any."""
from pathlib import Path

import numpy as np
import pytest

from tests.gpu_util import dev, host, sync

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def gpu_sample(cuda, rows, temp, top_p, top_k, us):
    torch = pytest.importorskip("torch")
    rows = np.ascontiguousarray(rows, np.float32)
    nrows, n = rows.shape
    ld, ud = dev(rows), dev(np.asarray(us, np.float32))
    tok = torch.empty(nrows, dtype=torch.int32, device="cuda")
    sync(cuda)
    cuda.sample(ld.data_ptr(), n, nrows, temp, top_p, top_k, ud.data_ptr(), tok.data_ptr())
    cuda.synchronize()
    return host(tok).astype(np.int64)


def test_sample_golden(cuda):
    from tests.golden.gen_golden import sample_logits
    g = np.load(GOLDEN / "sample.npz")
    vocab = int(g["vocab"])
    rows = {}
    for seed, temp, top_p, top_k, _rseed, u, tok in g["cases"]:
        seed = int(seed)
        if seed not in rows:
            rows[seed] = sample_logits(seed, vocab)
        got = gpu_sample(cuda, rows[seed][None, :], float(temp), float(top_p), int(top_k), [float(u)])
        assert got[0] == int(tok), (seed, temp, top_p, top_k, u)


CASES = [(0.0, 1.0, 0), (1.0, 1.0, 0), (0.7, 0.9, 40), (1.3, 0.5, 0), (1.0, 1.0, 1), (0.8, 1.0, 50),
         (1.0, 0.95, 0), (2.0, 0.3, 1000), (0.5, 1.0, 7)]


@pytest.mark.parametrize("temp,top_p,top_k", CASES)
def test_sample_rows_vs_oracle(temp, top_p, top_k, cuda, oracle):
    rng = np.random.Generator(np.random.PCG64(808))
    n, nrows = 50000, 6
    rows = (rng.standard_normal((nrows, n)) * 2.0).astype(np.float32)
    rows[1] = np.round(rows[1] * 2) / 2  # heavy ties: lower index first within a tie
    rows[2, :] = 0.25  # one value everywhere: the whole row is one tie
    rows[3, rng.integers(0, n, 40)] = rows[3].max()  # tied maxima
    rows[4] = rows[4] * 0.01  # nearly flat: the mass spreads over the whole row
    us = [0.0, 0.37, 0.999, 0.5, 0.71, 0.123]
    got = gpu_sample(cuda, rows, temp, top_p, top_k, us)
    for r in range(nrows):
        want = oracle.sample(rows[r], temp, top_p, top_k, us[r])
        assert got[r] == want, (r, got[r], want)
