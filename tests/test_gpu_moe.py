"""GPU parity of the routed MoE FFN (qw6cu_moe_decode) against the oracle's
composition of qw6_apply_layer_moe (qw6.c:2246-2264) and the golden fixture.
Routing indices must match exactly; outputs within 1e-3 max relative error."""

import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.conftest import rel_err, same_bits
from tests.gpu_util import dev, empty_f32, host, pack, sync
from tests.test_golden import golden_moe_weights

pytestmark = pytest.mark.gpu
TOL = 1e-3


def run_moe(cuda, gq, gate, up, dq, down, logits, x, top_k):
    E, I, H = gate.shape[0], gate.shape[1], x.shape[1]
    T = x.shape[0]
    pg, sg = pack(cuda, gq, gate, I, H, E)
    pu, su = pack(cuda, gq, up, I, H, E)
    pd, sd = pack(cuda, dq, down, H, I, E)
    ld, xd = dev(logits), dev(x)
    out = empty_f32(T, H)
    sync(cuda)
    cuda.moe_decode(L.ExpertPack(gq, pg.data_ptr(), sg), L.ExpertPack(gq, pu.data_ptr(), su),
                    L.ExpertPack(dq, pd.data_ptr(), sd), ld.data_ptr(), xd.data_ptr(), out.data_ptr(), T, H, I, E,
                    top_k)
    cuda.synchronize()
    return host(out)


def test_moe_golden_small(cuda):
    g, (E, H, I, K, T), (gate, up, down) = golden_moe_weights()
    out = run_moe(cuda, S.Q4_K, gate, up, S.Q6_K, down, g["logits"], g["x"], K)
    for t in range(T):
        assert rel_err(out[t], g["out"][t]) <= TOL


@pytest.mark.parametrize("ntok", [1, 2, 3, 4, 5, 8, 17])
def test_moe_small_experts_various_batches(ntok, cuda, oracle, rng):
    E, H, I, K = 16, 2048, 512, 8
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((ntok, E), dtype=np.float32)
    x = rng.standard_normal((ntok, H), dtype=np.float32)
    out = run_moe(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, x, K)
    ref, _, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=K)
    for t in range(ntok):
        assert rel_err(out[t], ref[t]) <= TOL, t


def test_moe_config1_decode(cuda, oracle):
    """Config 1: 256 experts, top-8, Q4_K gate/up, Q6_K down, one token."""
    gate, up, down, logits, x = S.config1()
    out = run_moe(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, x, 8)
    ref, idx, w = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=8)
    ref64 = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=8, f64=True)
    assert rel_err(out[0], ref[0]) <= TOL
    assert rel_err(out[0], ref64[0]) <= TOL


def test_moe_decode_ring_recycles(cuda, oracle, rng):
    """4 tokens over 256 experts: up to 32 distinct experts, so every
    gate/up CTA streams several (expert, row-tile) units through its
    shared-memory ring and reuses its slots."""
    E, H, I, K, T = 256, 2048, 512, 8, 4
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    out = run_moe(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, x, K)
    ref, idx, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=K)
    assert len(np.unique(idx)) > 24
    for t in range(T):
        assert rel_err(out[t], ref[t]) <= TOL, t


@pytest.mark.parametrize("H,I", [(1024, 2048), (2048, 1024)])
def test_moe_decode_other_shapes(H, I, cuda, oracle, rng):
    """inter 2048: the down kernel stages mid rows two experts at a time;
    hidden 1024 / inter 1024: other K-split and tile counts."""
    E, K, T = 16, 8, 2
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    out = run_moe(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, x, K)
    ref, _, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=K)
    for t in range(T):
        assert rel_err(out[t], ref[t]) <= TOL, t


def test_moe_config2_batched_iq2xxs(cuda, oracle):
    """Config 2: 64 tokens, IQ2_XXS experts."""
    gate, up, down, logits, x = S.config2()
    out = run_moe(cuda, S.IQ2_XXS, gate, up, S.IQ2_XXS, down, logits, x, 8)
    ref, _, _ = oracle.moe_layer(S.IQ2_XXS, gate, up, S.IQ2_XXS, down, logits, x, top_k=8)
    errs = [rel_err(out[t], ref[t]) for t in range(x.shape[0])]
    assert max(errs) <= TOL, max(errs)


def test_moe_rejects_mixed_gate_up_quant(cuda):
    with pytest.raises(L.Qw6CudaError):
        cuda.moe_decode(L.ExpertPack(S.Q4_K, 16, 0), L.ExpertPack(S.Q5_K, 16, 0), L.ExpertPack(S.Q6_K, 16, 0),
                        16, 16, 16, 1, 2048, 512, 8, 8)


@pytest.mark.parametrize("ntok", [1, 3, 6])
def test_moe_duplicate_expert_selection(ntok, cuda, oracle, rng):
    """All logits -inf except two: qw6's scan then re-selects expert 0 for the
    remaining slots (the winner is set to -inf, not removed); the same expert
    appears in several slots of one token and its output is summed per slot."""
    E, H, I, K = 16, 2048, 512, 8
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = np.full((ntok, E), -np.inf, np.float32)
    logits[:, 5] = 1.0
    logits[:, 9] = 0.5
    x = rng.standard_normal((ntok, H), dtype=np.float32)
    out = run_moe(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, x, K)
    ref, idx, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=K)
    assert list(idx[0]) == [5, 9, 0, 0, 0, 0, 0, 0]
    for t in range(ntok):
        assert rel_err(out[t], ref[t]) <= TOL, t


def test_moe_hidden_4096(cuda, oracle, rng):
    E, H, I, K, T = 8, 4096, 512, 4, 2
    gate, up, down = S.moe_weights(rng, E, S.Q5_K, S.IQ3_S, H, I)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    out = run_moe(cuda, S.Q5_K, gate, up, S.IQ3_S, down, logits, x, K)
    ref, _, _ = oracle.moe_layer(S.Q5_K, gate, up, S.IQ3_S, down, logits, x, top_k=K)
    for t in range(T):
        assert rel_err(out[t], ref[t]) <= TOL, t


@pytest.mark.parametrize("gq,dq", [(S.IQ2_S, S.Q4_K), (S.IQ2_XXS, S.IQ2_XXS), (S.Q6_K, S.Q5_K)])
def test_moe_format_mixes(gq, dq, cuda, oracle, rng):
    E, H, I, K, T = 12, 2048, 512, 4, 3
    gate, up, down = S.moe_weights(rng, E, gq, dq, H, I)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    out = run_moe(cuda, gq, gate, up, dq, down, logits, x, K)
    ref, _, _ = oracle.moe_layer(gq, gate, up, dq, down, logits, x, top_k=K)
    for t in range(T):
        assert rel_err(out[t], ref[t]) <= TOL, t


@pytest.mark.parametrize("ntok", [1, 12])
def test_moe_decode_hostio(ntok, cuda, oracle, rng):
    """qw6cu_moe_decode_hostio with host buffers, page-locked and pageable,
    gives qw6cu_moe_decode's bits on the two-launch path (1 token) and the
    planned one (12 tokens), also when a call reuses the context's buffers."""
    torch = pytest.importorskip("torch")
    E, H, I, K = 32, 2048, 512, 8
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((ntok, E), dtype=np.float32)
    x = rng.standard_normal((ntok, H), dtype=np.float32)
    want = run_moe(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, x, K)
    pg, sg = pack(cuda, S.Q4_K, gate, I, H, E)
    pu, su = pack(cuda, S.Q4_K, up, I, H, E)
    pd, sd = pack(cuda, S.Q6_K, down, H, I, E)
    packs = (L.ExpertPack(S.Q4_K, pg.data_ptr(), sg), L.ExpertPack(S.Q4_K, pu.data_ptr(), su),
             L.ExpertPack(S.Q6_K, pd.data_ptr(), sd))
    sync(cuda)
    h_lg, h_x = torch.from_numpy(logits).pin_memory(), torch.from_numpy(x).pin_memory()
    for _ in range(2):  # the second call reuses the context's buffers
        h_out = torch.full((ntok, H), float("nan")).pin_memory()
        cuda.moe_decode_hostio(*packs, h_lg.data_ptr(), h_x.data_ptr(), h_out.data_ptr(), ntok, H, I, E, K)
        assert same_bits(h_out.numpy(), want)
    p_out = np.full((ntok, H), np.nan, np.float32)
    cuda.moe_decode_hostio(*packs, logits.ctypes.data, x.ctypes.data, p_out.ctypes.data, ntok, H, I, E, K)
    assert same_bits(p_out, want)
    ref, _, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=K)
    assert max(rel_err(want[t], ref[t]) for t in range(ntok)) <= TOL
