"""GPU parity of the tensor-core prefill MoE (qw6cu_moe_prefill) against the
oracle's fp32 composition of qw6_apply_layer_moe (qw6.c:2246-2264) on the
same bf16-exact activations.  Tolerance: max relative error 2e-2 (bf16
tensor-core prefill)."""
import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.conftest import rel_err, same_bits
from tests.gpu_util import dev, empty_f32, host, pack, sync

pytestmark = pytest.mark.gpu
TOL = 2e-2


def run_prefill(cuda, gq, gate, up, dq, down, logits, x_bf16_bits, top_k):
    E, I, H = gate.shape[0], gate.shape[1], x_bf16_bits.shape[1]
    T = x_bf16_bits.shape[0]
    pg, sg = pack(cuda, gq, gate, I, H, E)
    pu, su = pack(cuda, gq, up, I, H, E)
    pd, sd = pack(cuda, dq, down, H, I, E)
    ld, xd = dev(logits), dev(x_bf16_bits.view(np.int16))
    out = empty_f32(T, H)
    sync(cuda)
    cuda.moe_prefill(L.ExpertPack(gq, pg.data_ptr(), sg), L.ExpertPack(gq, pu.data_ptr(), su),
                     L.ExpertPack(dq, pd.data_ptr(), sd), ld.data_ptr(), xd.data_ptr(), out.data_ptr(), T, H, I, E,
                     top_k)
    cuda.check_device_errors()
    return host(out)


def check_tokens(oracle, gq, gate, up, dq, down, logits, xbits, out, tokens, top_k):
    """Max relative error of the sampled tokens against the fp32 oracle and
    against its float64 recomputation (which shows the fp32 oracle's own
    accumulation-order noise); both within the bf16 prefill tolerance."""
    x32 = S.bf16_to_f32(xbits)
    ref, _, _ = oracle.moe_layer(gq, gate, up, dq, down, logits[tokens], x32[tokens], top_k=top_k)
    ref64 = oracle.moe_layer(gq, gate, up, dq, down, logits[tokens], x32[tokens], top_k=top_k, f64=True)
    errs = [rel_err(out[t], ref[i]) for i, t in enumerate(tokens)]
    errs64 = [rel_err(out[t], ref64[i]) for i, t in enumerate(tokens)]
    assert max(errs) <= TOL, max(errs)
    assert max(errs64) <= TOL, max(errs64)
    return max(errs)


@pytest.mark.parametrize("T", [1, 37, 300])
def test_prefill_small(T, cuda, oracle, rng):
    E, H, I, K = 16, 2048, 512, 8
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    xbits = S.bf16_round(rng.standard_normal((T, H), dtype=np.float32))
    out = run_prefill(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, xbits, K)
    toks = list(range(T)) if T <= 40 else list(rng.choice(T, 40, replace=False))
    check_tokens(oracle, S.Q4_K, gate, up, S.Q6_K, down, logits, xbits, out, toks, K)


def test_prefill_imbalanced_multi_chunk(cuda, oracle, rng):
    """Biased routing: some experts get > 256 tokens (several work items)."""
    E, H, I, K, T = 32, 2048, 512, 8, 1500
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    bias = np.zeros(E, np.float32)
    bias[[3, 7]] = 4.0
    logits = rng.standard_normal((T, E), dtype=np.float32) + bias
    xbits = S.bf16_round(rng.standard_normal((T, H), dtype=np.float32))
    out = run_prefill(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, xbits, K)
    toks = list(rng.choice(T, 48, replace=False))
    check_tokens(oracle, S.Q4_K, gate, up, S.Q6_K, down, logits, xbits, out, toks, K)


def test_prefill_q6k_gate_q4k_down(cuda, oracle, rng):
    E, H, I, K, T = 8, 2048, 512, 4, 64
    gate, up, down = S.moe_weights(rng, E, S.Q6_K, S.Q4_K, H, I)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    xbits = S.bf16_round(rng.standard_normal((T, H), dtype=np.float32))
    out = run_prefill(cuda, S.Q6_K, gate, up, S.Q4_K, down, logits, xbits, K)
    check_tokens(oracle, S.Q6_K, gate, up, S.Q4_K, down, logits, xbits, out, list(range(0, T, 3)), K)


def test_prefill_config3(cuda, oracle, rng):
    """Config 3: 4096 tokens, 256 experts, per-expert logit bias N(0, 0.5).
    Every token is checked against the oracle's expert-grouped float64
    recomputation (bit-exact routing and dequantized weights), and a seeded
    sample of 256 tokens against the fp32 oracle (qw6's own evaluation
    order)."""
    gate, up, down, logits, xbits = S.config3()
    out = run_prefill(cuda, S.Q4_K, gate, up, S.Q6_K, down, logits, xbits, 8)
    x32 = S.bf16_to_f32(xbits)
    ref64, _, _ = oracle.moe_layer_grouped_f64(S.Q4_K, gate, up, S.Q6_K, down, logits, x32, top_k=8)
    errs = [rel_err(out[t], ref64[t]) for t in range(out.shape[0])]
    assert max(errs) <= TOL, (int(np.argmax(errs)), max(errs))
    toks = list(np.random.Generator(np.random.PCG64(33)).choice(4096, 256, replace=False))
    ref, _, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits[toks], x32[toks], top_k=8)
    errs32 = [rel_err(out[t], ref[i]) for i, t in enumerate(toks)]
    assert max(errs32) <= TOL, max(errs32)


def test_prefill_hostio_pipelined(cuda, oracle, rng):
    """qw6cu_moe_prefill_hostio: batches in host memory, pipelined over two
    device slots (copy-in of batch b+1 and read-back of b-1 beside the experts
    of b).  Five batches from page-locked memory (one repeated, so both slots
    are reused) and two from pageable numpy arrays: every output is bit for bit
    qw6cu_moe_prefill's on the same batch, and sampled tokens are within the
    prefill tolerance of the fp32 oracle."""
    torch = pytest.importorskip("torch")
    E, H, I, K, T = 32, 2048, 512, 8, 300
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    pg, sg = pack(cuda, S.Q4_K, gate, I, H, E)
    pu, su = pack(cuda, S.Q4_K, up, I, H, E)
    pd, sd = pack(cuda, S.Q6_K, down, H, I, E)
    packs = (L.ExpertPack(S.Q4_K, pg.data_ptr(), sg), L.ExpertPack(S.Q4_K, pu.data_ptr(), su),
             L.ExpertPack(S.Q6_K, pd.data_ptr(), sd))
    lgs = [rng.standard_normal((T, E), dtype=np.float32) for _ in range(4)]
    xbs = [S.bf16_round(rng.standard_normal((T, H), dtype=np.float32)) for _ in range(4)]
    # device reference: one qw6cu_moe_prefill per distinct batch
    ref = []
    for lg, xb in zip(lgs, xbs):
        ld, xd = dev(lg), dev(xb.view(np.int16))
        o = empty_f32(T, H)
        sync(cuda)
        cuda.moe_prefill(*packs, ld.data_ptr(), xd.data_ptr(), o.data_ptr(), T, H, I, E, K)
        cuda.check_device_errors()
        ref.append(host(o))
    order = [0, 1, 2, 3, 1]
    h_lg = [torch.from_numpy(lg).pin_memory() for lg in lgs]
    h_x = [torch.from_numpy(xb.view(np.int16)).pin_memory() for xb in xbs]
    h_out = [torch.full((T, H), float("nan"), dtype=torch.float32).pin_memory() for _ in order]
    sync(cuda)
    cuda.moe_prefill_hostio(*packs, [h_lg[b].data_ptr() for b in order], [h_x[b].data_ptr() for b in order],
                            [o.data_ptr() for o in h_out], T, H, I, E, K)
    cuda.check_device_errors()
    for o, b in zip(h_out, order):
        assert same_bits(o.numpy(), ref[b]), b
    # pageable host memory: same results, copies serialized
    p_lg = [np.ascontiguousarray(lgs[b]) for b in (2, 0)]
    p_x = [np.ascontiguousarray(xbs[b]) for b in (2, 0)]
    p_out = [np.full((T, H), np.nan, np.float32) for _ in range(2)]
    cuda.moe_prefill_hostio(*packs, [a.ctypes.data for a in p_lg], [a.ctypes.data for a in p_x],
                            [a.ctypes.data for a in p_out], T, H, I, E, K)
    assert same_bits(p_out[0], ref[2]) and same_bits(p_out[1], ref[0])
    toks = list(rng.choice(T, 24, replace=False))
    check_tokens(oracle, S.Q4_K, gate, up, S.Q6_K, down, lgs[3], xbs[3], h_out[3].numpy(), toks, K)
    # no batches: nothing to do; a null host buffer: rejected before any copy
    cuda.moe_prefill_hostio(*packs, [], [], [], T, H, I, E, K)
    with pytest.raises(L.Qw6CudaError, match="null host buffer of batch 1"):
        cuda.moe_prefill_hostio(*packs, [h_lg[0].data_ptr()] * 2, [h_x[0].data_ptr(), 0],
                                [o.data_ptr() for o in h_out[:2]], T, H, I, E, K)
