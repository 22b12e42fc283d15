"""GPU parity of the fused LM head + greedy argmax (config 4's Q6_K output
projection, qw6.c:2493 + qw6_cpu_argmax qw6.c:2858-2863), whole and row-sharded."""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from qw6_b200 import synth as S
from tests.conftest import rel_err
from tests.gpu_util import dev, empty_f32, host, pack, sync

pytestmark = pytest.mark.gpu


def lm_head(cuda, quant, w, x, rows, cols, shards=1, want_logits=False):
    torch = pytest.importorskip("torch")
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    ntok = x.shape[0]
    xd = dev(x)
    keys = torch.zeros((shards, ntok), dtype=torch.int64, device="cuda")
    logits = empty_f32(ntok, rows) if want_logits else None
    bounds = np.linspace(0, rows, shards + 1).astype(int)
    bounds[1:-1] = bounds[1:-1] // 16 * 16
    held = []
    for s in range(shards):
        r0, r1 = int(bounds[s]), int(bounds[s + 1])
        rb = w.shape[1]
        pk, _ = pack(cuda, quant, w[r0:r1], r1 - r0, cols)
        held.append(pk)
        sync(cuda)
        lg = None
        if want_logits and shards == 1:
            lg = logits.data_ptr()
        cuda.lm_head_argmax(quant, pk.data_ptr(), xd.data_ptr(), ntok, r1 - r0, cols, r0,
                            keys[s].data_ptr(), lg)
        cuda.synchronize()
        del rb
    idx = torch.empty(ntok, dtype=torch.int32, device="cuda")
    val = empty_f32(ntok)
    cuda.argmax_keys_reduce(keys.data_ptr(), shards, ntok, idx.data_ptr(), val.data_ptr())
    cuda.synchronize()
    return host(idx), host(val), (host(logits) if want_logits else None)


@pytest.mark.parametrize("q", [S.Q6_K, S.Q4_K, S.IQ2_XXS])
@pytest.mark.parametrize("ntok", [1, 3, 32])
def test_lm_head_argmax_vs_oracle(q, ntok, cuda, oracle, rng):
    rows, cols = 5003, 2048
    w = S.make_matrix(q, rows, cols, rng)
    x = rng.standard_normal((ntok, cols), dtype=np.float32)
    idx, val, lg = lm_head(cuda, q, w, x, rows, cols, want_logits=True)
    ref = oracle.matvec(q, w, x, rows, cols).reshape(ntok, rows)
    for t in range(ntok):
        assert idx[t] == oracle.argmax(ref[t])
        assert abs(val[t] - ref[t][idx[t]]) <= 1e-3 * np.max(np.abs(ref[t]))
        assert rel_err(lg[t], ref[t]) <= 1e-3
        assert idx[t] == int(np.argmax(lg[t]))


@pytest.mark.parametrize("shards,rows", [(2, 4096), (3, 4096), (8, 4096), (2, 37888), (8, 37888)])
def test_lm_head_row_shards_combine_exactly(shards, rows, cuda, rng):
    """Row shards give the whole vocabulary's bits; 37888 rows is where a
    split factor chosen by row count would differ between whole and shards."""
    cols, ntok = 2048, 5
    w = S.make_matrix(S.Q6_K, rows, cols, rng)
    x = rng.standard_normal((ntok, cols), dtype=np.float32)
    i1, v1, _ = lm_head(cuda, S.Q6_K, w, x, rows, cols, shards=1)
    i2, v2, _ = lm_head(cuda, S.Q6_K, w, x, rows, cols, shards=shards)
    assert np.array_equal(i1, i2) and np.array_equal(v1.view(np.uint32), v2.view(np.uint32))


def test_lm_head_ties_lowest_index(cuda, rng):
    """Identical rows give identical logits; the lowest index must win."""
    rows, cols = 512, 2048
    w = S.make_matrix(S.Q6_K, rows, cols, rng)
    x = rng.standard_normal(cols, dtype=np.float32)
    idx0, _, lg = lm_head(cuda, S.Q6_K, w, x, rows, cols, want_logits=True)
    top = int(idx0[0])
    w2 = w.copy()
    for r in (3, 100, 400):
        w2[r] = w[top]
    idx, _, _ = lm_head(cuda, S.Q6_K, w2, x, rows, cols, shards=4)
    assert int(idx[0]) == min(3, top)


def test_lm_head_config4_vocab(cuda, reference, rng):
    """Full Q6_K LM head [248320 x 2048], batch 1: argmax equals qw6's CPU
    qw6_tensor_matvec + qw6_cpu_argmax (oracle/_ref), row-sharded 8 ways."""
    rows, cols = S.VOCAB, 2048
    w = S.make_matrix(S.Q6_K, rows, cols, rng)
    x = rng.standard_normal(cols, dtype=np.float32)
    nth = 8
    bounds = np.linspace(0, rows, nth + 1).astype(int)
    with ThreadPoolExecutor(nth) as ex:
        parts = list(ex.map(lambda i: reference.matvec(S.Q6_K, w[bounds[i]:bounds[i + 1]], x,
                                                       int(bounds[i + 1] - bounds[i]), cols), range(nth)))
    ref = np.concatenate(parts)
    idx, val, _ = lm_head(cuda, S.Q6_K, w, x, rows, cols, shards=8)
    assert int(idx[0]) == reference.argmax(ref)
    assert abs(val[0] - ref[idx[0]]) <= 1e-3 * np.max(np.abs(ref))
