"""CPU: the oracle reproduces the committed fixtures made by qw6's own code
(tests/golden/gen_golden.py).  These run without the reference tree."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from qw6_b200 import synth as S
from tests.conftest import same_bits

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("name", [S.QUANT_NAMES[q] for q in S.BLOCK_QUANTS])
def test_golden_matvec(name, oracle):
    g = np.load(GOLDEN / f"matvec_{name}.npz")
    q, rows, cols = int(g["quant"]), int(g["rows"]), int(g["cols"])
    assert same_bits(oracle.dequantize(q, g["w"], rows, cols), g["deq"])
    assert same_bits(oracle.matvec(q, g["w"], g["x"], rows, cols), g["y"])
    ns = g["w_special"].shape[0]
    assert same_bits(oracle.dequantize(q, g["w_special"], ns, cols), g["deq_special"])


def test_golden_route(oracle):
    g = np.load(GOLDEN / "route.npz")
    for lg, idx, w in zip(g["logits"], g["idx"], g["w"]):
        i, ww = oracle.moe_route(lg, 8)
        assert np.array_equal(i, idx) and same_bits(ww, w)


def test_golden_argmax(oracle):
    g = np.load(GOLDEN / "argmax.npz")
    for x, n, idx in zip(g["x"], g["n"], g["idx"]):
        assert oracle.argmax(x[:n]) == idx


def golden_moe_weights():
    g = np.load(GOLDEN / "moe_small.npz")
    E, H, I, K, T = (int(v) for v in g["dims"])
    rng = np.random.Generator(np.random.PCG64(int(g["seed"])))
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    sha = hashlib.sha256(gate.tobytes() + up.tobytes() + down.tobytes()).hexdigest()
    assert sha == str(g["sha"]), "synthetic generator drifted from the fixture"
    return g, (E, H, I, K, T), (gate, up, down)


def test_golden_moe(oracle):
    g, (E, H, I, K, T), (gate, up, down) = golden_moe_weights()
    out, idx, w = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, g["logits"], g["x"], top_k=K)
    assert np.array_equal(idx, g["idx"]) and same_bits(w, g["w"])
    assert same_bits(out, g["out"])


def test_golden_moe_block(oracle):
    """The full MoE FFN block against qw6's own composition (with and
    without the shared expert); inputs regenerated from the fixture's seed."""
    from tests.golden.gen_golden import block_inputs
    g = np.load(GOLDEN / "moe_block.npz")
    b = block_inputs(int(g["seed"]))
    assert b["sha"] == str(g["sha"]), "synthetic generator drifted from the fixture"
    K = b["dims"][4]
    out = oracle.moe_block(b["x"], b["norm_w"], b["router"], b["experts"], b["shared"], top_k=K)
    assert same_bits(out, g["out"])
    routed = oracle.moe_block(b["x"], b["norm_w"], b["router"], b["experts"], None, top_k=K)
    assert same_bits(routed, g["out_routed"])


def test_golden_sample(oracle):
    """qw6_sample's picks (with the uniform draw each made) on logit rows
    regenerated from the fixture's seeds."""
    from tests.golden.gen_golden import sample_logits
    g = np.load(GOLDEN / "sample.npz")
    vocab = int(g["vocab"])
    assert hashlib.sha256(sample_logits(300, vocab).tobytes()).hexdigest() == str(g["sha"])
    rows = {}
    for seed, temp, top_p, top_k, _rseed, u, tok in g["cases"]:
        seed = int(seed)
        if seed not in rows:
            rows[seed] = sample_logits(seed, vocab)
        assert oracle.sample(rows[seed], float(temp), float(top_p), int(top_k), float(u)) == int(tok)
    assert len({int(t) for t in g["cases"][:, 6]}) > 3  # the picks are not all the same token
