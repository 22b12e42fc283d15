"""The forward-pass checker (oracle/qw6_oracle_fwd.c) against qw6's own
forward pass (qw6_forward_token, qw6.c:2426-2500, compiled from its sources
into oracle/_ref): bit-identical logits over two positions of a seeded
40-layer model, so the DeltaNet state, the conv window and the KV cache carry
from one token to the next.  Plus the checker's own error behaviour."""
import threading

import numpy as np
import pytest

from qw6_b200 import synth as S


def _both(fa, fb):
    """Run two ctypes-bound calls at once (they release the GIL)."""
    out = {}

    def run(k, f):
        out[k] = f()

    ts = [threading.Thread(target=run, args=(k, f)) for k, f in (("a", fa), ("b", fb))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    return out["a"], out["b"]


def test_forward_matches_qw6(oracle, reference):
    m = S.fwd_model(seed=11, n_layers=40, vocab=2048, embd_rows=1024)
    tokens = [7, 300]
    got, want = _both(lambda: oracle.forward(m, tokens), lambda: reference.forward(m, tokens))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.isfinite(got).all() and np.abs(got).max() > 0


def test_forward_state_carries(oracle):
    """The second token's logits depend on the first token (recurrent state
    and cache), and a repeated run from a cleared state repeats them."""
    m = S.fwd_model(seed=12, n_layers=4, vocab=1024, embd_rows=256)
    a = oracle.forward(m, [5, 9])
    b = oracle.forward(m, [6, 9])
    c = oracle.forward(m, [5, 9])
    assert not np.array_equal(a[1], b[1])
    assert np.array_equal(a, c)


def test_forward_rejects_bad_input(oracle):
    m = S.fwd_model(seed=13, n_layers=4, vocab=512, embd_rows=64)
    with pytest.raises(ValueError):
        oracle.forward(m, [64])  # past the embedding rows
    # a NaN in the hidden state ends the step with an error, as qw6's check does (qw6.c:2457)
    f, l, q, r, c, arr, st = next(t for t in m.tensors if t[0] == S.F_NORM and t[1] == 2)
    bad = arr.copy()
    bad[0, 0] = np.nan
    m.tensors = [t if not (t[0] == S.F_NORM and t[1] == 2) else (f, l, q, r, c, bad, st) for t in m.tensors]
    with pytest.raises(ValueError):
        oracle.forward(m, [3])
