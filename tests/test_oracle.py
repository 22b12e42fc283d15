"""CPU: the oracle restatement is pinned to qw6's own compiled CPU code
(oracle/_ref), to the committed golden fixtures and to closed-form KATs."""
import numpy as np
import pytest

from qw6_b200 import synth as S
from tests.conftest import same_bits

SPECIAL_D = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x7E00, 0x3C00, 0xBC00]


def d_offset(q):
    return 208 if q == S.Q6_K else 0


def special_matrix(q, rng):
    """Rows whose fp16 scales cover zero, subnormal, max, +-inf and NaN."""
    rows, cols = len(SPECIAL_D), 512
    w = S.make_matrix(q, rows, cols, rng)
    nb, bb = cols // 256, S.BLOCK_BYTES[q]
    blocks = w.reshape(rows, nb, bb)
    for r, d in enumerate(SPECIAL_D):
        o = d_offset(q)
        blocks[r, :, o] = d & 0xFF
        blocks[r, :, o + 1] = d >> 8
        if q in (S.Q4_K, S.Q5_K):  # dmin as well
            blocks[r, :, 2] = d & 0xFF
            blocks[r, :, 3] = d >> 8
    return w, rows, cols


@pytest.mark.parametrize("q", S.BLOCK_QUANTS)
def test_dequant_matches_reference_bitexact(q, oracle, reference, rng):
    for rows, cols in [(1, 256), (7, 512), (16, 2048), (3, 4096)]:
        w = S.make_matrix(q, rows, cols, rng)
        assert same_bits(oracle.dequantize(q, w, rows, cols), reference.dequantize(q, w, rows, cols))


@pytest.mark.parametrize("q", S.BLOCK_QUANTS)
def test_dequant_special_scales_bitexact(q, oracle, reference, rng):
    w, rows, cols = special_matrix(q, rng)
    assert same_bits(oracle.dequantize(q, w, rows, cols), reference.dequantize(q, w, rows, cols))


@pytest.mark.parametrize("q", S.BLOCK_QUANTS)
def test_matvec_matches_reference_bitexact(q, oracle, reference, rng):
    for rows, cols in [(5, 256), (33, 2048)]:
        w = S.make_matrix(q, rows, cols, rng)
        x = rng.standard_normal(cols, dtype=np.float32)
        assert same_bits(oracle.matvec(q, w, x, rows, cols), reference.matvec(q, w, x, rows, cols))


@pytest.mark.parametrize("q", [S.FP16, S.BF16])
def test_dequant16_matches_reference_bitexact(q, oracle, reference, rng):
    """FP16 / BF16 rows, including every class of special value, widen to the
    same bits as qw6_tensor_dequantize_row (qw6.c:1686-1692)."""
    rows, cols = 6, 512
    h = rng.integers(0, 1 << 16, size=(rows, cols), dtype=np.uint16)
    w = h.view(np.uint8).reshape(rows, cols * 2)
    assert same_bits(oracle.dequantize(q, w, rows, cols), reference.dequantize(q, w, rows, cols))


def test_fp16_exhaustive(oracle):
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.fp16_to_f32(int(v)) for v in h], np.float32)
    assert same_bits(got, ref)


def test_route_matches_reference_with_ties(oracle, reference, rng):
    for t in range(300):
        lg = rng.standard_normal(256).astype(np.float32)
        if t % 3 == 0:
            lg[rng.integers(0, 256, 6)] = lg.max()
        if t % 5 == 0:
            lg = np.round(lg * 2) / 2  # many ties
        k = 1 + t % 8
        i1, w1 = oracle.moe_route(lg, k)
        i2, w2 = reference.moe_route(lg, k)
        assert np.array_equal(i1, i2)
        assert same_bits(w1, w2)


def test_route_cpu_kat(oracle):
    # qw6.c:3400-3412: logits {0,2,1,-1}, top-2 -> {1,2}, weights sum to 1.
    idx, w = oracle.moe_route(np.array([0, 2, 1, -1], np.float32), 2)
    assert list(idx) == [1, 2]
    assert abs(float(w.sum()) - 1.0) < 1e-6 and w[0] >= w[1]


def test_route_edge_values(oracle, reference):
    cases = [np.full(256, -np.inf, np.float32), np.zeros(256, np.float32)]
    lg = np.full(256, -np.inf, np.float32)
    lg[[3, 9, 200]] = [1.0, 2.0, 3.0]
    cases.append(lg)
    lg = np.linspace(-1, 1, 256).astype(np.float32)
    lg[0] = np.nan
    cases.append(lg)
    lg = np.linspace(-1, 1, 256).astype(np.float32)
    lg[17] = np.nan
    cases.append(lg)
    for lg in cases:
        i1, w1 = oracle.moe_route(lg, 8)
        i2, w2 = reference.moe_route(lg, 8)
        assert np.array_equal(i1, i2)
        assert same_bits(w1, w2)


def test_argmax_ties_and_nan(oracle, reference):
    x = np.array([1, 5, 5, 2, 5], np.float32)
    assert oracle.argmax(x) == reference.argmax(x) == 1
    x = np.array([np.nan, 1, 2], np.float32)
    assert oracle.argmax(x) == reference.argmax(x) == 0
    x = np.array([0, np.nan, 2, 2], np.float32)
    assert oracle.argmax(x) == reference.argmax(x) == 2
    x = np.full(10, -np.inf, np.float32)
    assert oracle.argmax(x) == reference.argmax(x) == 0


def test_silu_matches_reference(oracle, reference):
    v = np.linspace(-30, 30, 2001).astype(np.float32)
    got = oracle.silu_mul(v, np.ones_like(v))
    want = np.array([reference.silu(float(a)) for a in v], np.float32)
    assert same_bits(got, want)


def test_moe_layer_matches_reference_composition(oracle, reference, rng):
    """qo_moe_layer == qw6's functions composed as qw6.c:2246-2264."""
    E, H, I = 16, 512, 512
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((2, E), dtype=np.float32)
    x = rng.standard_normal((2, H), dtype=np.float32)
    o1, i1, w1 = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=4)
    o2, i2, w2 = reference.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=4)
    assert np.array_equal(i1, i2) and same_bits(w1, w2)
    assert same_bits(o1, o2)
    # the all-C token loop the CPU baseline times gives the same bits
    o3 = reference.moe_tokens(S.Q4_K, gate, up, S.Q6_K, down, logits, x, 0, 2, top_k=4)
    assert same_bits(o3, o2)
    assert same_bits(reference.moe_tokens(S.Q4_K, gate, up, S.Q6_K, down, logits, x, 1, 2, top_k=4), o2[1:])


def test_moe_layer_grouped_f64_matches_per_token_f64(oracle, rng):
    """The expert-grouped float64 recomputation used for whole-batch GPU
    checks agrees with the oracle's per-token float64 layer (same routing,
    same bit-exact weights) to float64 rounding."""
    E, H, I, T = 12, 512, 256, 9
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    g64, idx, w = oracle.moe_layer_grouped_f64(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=4)
    p64 = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=4, f64=True)
    _, i32, w32 = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=4)
    assert np.array_equal(idx, i32) and same_bits(w, w32)
    assert np.max(np.abs(g64 - p64)) <= 1e-12 * np.max(np.abs(p64))


# ---- known-answer tests of qw6's Vulkan self-test, against the oracle ----

def _q4k_kat():
    w = np.zeros((3, 144), np.uint8)
    x = np.sin(np.arange(256, dtype=np.float32) * np.float32(0.031)).astype(np.float32)
    want = np.zeros(3)
    for r in range(3):
        b = w[r]
        b[0:2] = [0x00, 0x3C]
        b[4:8] = 1
        b[12:16] = 1
        for c in range(256):
            chunk, hi, l = c // 64, (c // 32) & 1, c % 32
            q = (r * 3 + c * 5 + 7) & 15
            p = 16 + 32 * chunk + l
            b[p] = (b[p] & 0x0F) | (q << 4) if hi else (b[p] & 0xF0) | q
            want[r] += q * float(x[c])
    return w, x, want


def test_kat_q4k(oracle):
    w, x, want = _q4k_kat()
    assert np.max(np.abs(oracle.matvec(S.Q4_K, w, x, 3, 256) - want)) < 1e-2


def test_kat_iq2xxs(oracle):
    w = np.zeros((3, 66), np.uint8)
    for r, d in enumerate([0x3C00, 0x3E00, 0x4000]):
        w[r, 0], w[r, 1] = d & 0xFF, d >> 8
    x = (np.sin(np.arange(256) * 0.029) + 0.15 * np.cos(np.arange(256) * 0.017)).astype(np.float32)
    want = np.array([1.0, 1.5, 2.0]) * float(x.astype(np.float64).sum())
    assert np.max(np.abs(oracle.matvec(S.IQ2_XXS, w, x, 3, 256) - want)) < 2e-2


def test_kat_route_sin_cos(oracle, reference):
    i = np.arange(256, dtype=np.float32)
    lg = (np.sin(i * np.float32(0.17)) + np.cos(i * np.float32(0.031))).astype(np.float32)
    lg[7], lg[149] = 5.0, 4.5
    i1, w1 = oracle.moe_route(lg, 8)
    i2, w2 = reference.moe_route(lg, 8)
    assert i1[0] == 7 and i1[1] == 149
    assert np.array_equal(i1, i2) and np.max(np.abs(w1 - w2)) <= 2e-5


def _block_data(rng, E=16, H=512, I=256, SI=256, ntok=3):
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    router = (S.FP32, (rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.05)).astype(np.float32))
    shared = ((S.Q4_K, S.make_matrix(S.Q4_K, SI, H, rng)), (S.Q4_K, S.make_matrix(S.Q4_K, SI, H, rng)),
              (S.Q6_K, S.make_matrix(S.Q6_K, H, SI, rng)),
              (S.FP32, (rng.standard_normal((1, H), dtype=np.float32) * np.float32(0.05)).astype(np.float32)))
    norm_w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    x = rng.standard_normal((ntok, H), dtype=np.float32)
    return x, norm_w, router, (S.Q4_K, gate, up, S.Q6_K, down), shared


@pytest.mark.parametrize("variant", ["shared_gated", "shared_ungated", "routed_only"])
def test_moe_block_matches_reference_bitexact(variant, oracle, reference, rng):
    """The full MoE FFN block (rmsnorm, router matvec, routed experts,
    shared expert with its sigmoid gate, residual add) restated in C equals
    qw6's own functions composed in qw6's order, bit for bit."""
    x, norm_w, router, experts, shared = _block_data(rng)
    if variant == "shared_ungated":
        shared = shared[:3] + (None,)
    elif variant == "routed_only":
        shared = None
    got = oracle.moe_block(x, norm_w, router, experts, shared, top_k=4)
    want = reference.moe_block(x, norm_w, router, experts, shared, top_k=4)
    assert same_bits(got, want)
    assert np.all(np.isfinite(got))


def test_rmsnorm_matches_reference_bitexact(oracle, reference, rng):
    for dim in (1, 7, 512, 2048):
        x = (rng.standard_normal(dim) * 10.0 ** rng.uniform(-3, 3)).astype(np.float32)
        w = rng.standard_normal(dim).astype(np.float32)
        assert same_bits(oracle.rmsnorm(x, w), reference.rmsnorm(x, w))


def test_moe_block_shared_expert_contributes(oracle, rng):
    x, norm_w, router, experts, shared = _block_data(rng, ntok=2)
    routed = oracle.moe_block(x, norm_w, router, experts, None, top_k=4)
    gated = oracle.moe_block(x, norm_w, router, experts, shared, top_k=4)
    ungated = oracle.moe_block(x, norm_w, router, experts, shared[:3] + (None,), top_k=4)
    assert not np.array_equal(routed, gated) and not np.array_equal(gated, ungated)
    # the residual: with zero routed and shared weights the block returns x unchanged
    zero = tuple(np.zeros_like(m) for m in experts[1:3]) + (np.zeros_like(experts[4]),)
    z = oracle.moe_block(x, norm_w, router, (experts[0], zero[0], zero[1], experts[3], zero[2]), None, top_k=4)
    assert same_bits(z, x)


@pytest.mark.parametrize("shared_on", [True, False])
def test_moe_block_f64_error_reference(shared_on, oracle, rng):
    """The double-precision block routes like the fp32 one and differs from
    it only by fp32 accumulation noise."""
    x, norm_w, router, experts, shared = _block_data(rng)
    sh = shared if shared_on else None
    out32 = oracle.moe_block(x, norm_w, router, experts, sh, top_k=4)
    out64 = oracle.moe_block(x, norm_w, router, experts, sh, top_k=4, f64=True)
    assert out64.dtype == np.float64
    err = float(np.max(np.abs(out32 - out64)) / np.max(np.abs(out64)))
    assert 0 < err <= 1e-5, err


def test_sample_cpu_kat(oracle):
    """qw6's own sampling self-test (qw6.c:3369-3384)."""
    v = np.zeros(248320, np.float32)
    v[:3] = [1.0, 2.0, 3.0]
    assert oracle.sample(v, 0.0, 1.0, 0, 0.5) == 2
    assert oracle.sample(v, 1.0, 1.0, 1, 0.99) == 2
    v[:] = -100.0
    v[:3] = [10.0, 0.0, 0.0]
    assert oracle.sample(v, 1.0, 0.5, 0, 0.99) == 0


@pytest.mark.parametrize("temp,top_p,top_k", [(0.0, 1.0, 0), (1.0, 1.0, 0), (0.7, 0.9, 40), (1.3, 0.5, 0),
                                              (1.0, 1.0, 1), (0.8, 1.0, 50), (1.0, 0.95, 0), (2.0, 1.5, -3)])
def test_sample_matches_reference(temp, top_p, top_k, oracle, reference):
    """The sampler restated with its uniform draw given equals qw6_sample
    with libc rand() seeded to produce that draw (the full vocabulary row,
    with a few tied logits)."""
    rng = np.random.Generator(np.random.PCG64(int(temp * 10) + top_k + 100))
    logits = (rng.standard_normal(reference.vocab) * 3.0).astype(np.float32)
    logits[rng.integers(0, reference.vocab, 8)] = logits.max()
    for seed in (1, 7, 12345):
        u = reference.rand_unit(seed)
        assert oracle.sample(logits, temp, top_p, top_k, u) == reference.sample(logits, temp, top_p, top_k, seed)
