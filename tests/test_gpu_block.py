"""GPU parity of the MoE FFN block (qw6cu_moe_block: RMSNorm, fp32 router,
routed experts, shared expert with its sigmoid gate, residual -- qw6.c:2474-2484
around qw6_apply_layer_moe, qw6.c:2226-2290) against the oracle's block,
which is pinned bit for bit to qw6's own functions, and against the golden
fixture made by qw6's own code.  The FFN part (out - x) must be within 1e-3
max relative error of the oracle's and of its float64 recomputation.

The router's logits are fp32 like qw6's but summed in another order, so the
cases check first, on the CPU, that no token's k-th and (k+1)-th logits are
within rounding of each other (where the expert choice would be a coin
flip); the seeded inputs are chosen to pass that check."""
import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.conftest import rel_err
from tests.gpu_util import dev, empty_f32, host, pack, sync

pytestmark = pytest.mark.gpu
TOL = 1e-3


def routing_margin_ok(oracle, x, norm_w, router, top_k, rel=1e-4):
    for t in range(x.shape[0]):
        n = oracle.rmsnorm(x[t], norm_w)
        lg = router @ n.astype(np.float64)
        s = np.sort(lg)[::-1]
        if s[top_k - 1] - s[top_k] <= rel * max(1.0, abs(s[0])):
            return False
    return True


def run_block(cuda, x, norm_w, router, experts, shared, top_k):
    gq, gate, up, dq, down = experts
    E, I, H = gate.shape[0], gate.shape[1], x.shape[1]
    T = x.shape[0]
    keep = []
    pg, sgs = pack(cuda, gq, gate, I, H, E)
    pu, sus = pack(cuda, gq, up, I, H, E)
    pd, sds = pack(cuda, dq, down, H, I, E)
    keep += [pg, pu, pd]
    sh = None
    if shared is not None:
        (qg, mg), (qu, mu), (qd, md), srt = shared
        SI = mg.shape[0]
        tg, _ = pack(cuda, qg, mg, SI, H)
        tu, _ = pack(cuda, qu, mu, SI, H)
        td, _ = pack(cuda, qd, md, H, SI)
        keep += [tg, tu, td]
        rt = None
        if srt is not None:
            rt = dev(np.ascontiguousarray(srt[1], np.float32).reshape(-1))
            keep.append(rt)
        sh = L.SharedExpert(qg, qu, qd, tg.data_ptr(), tu.data_ptr(), td.data_ptr(), SI,
                            rt.data_ptr() if rt is not None else None)
    xd, wd, rd = dev(x), dev(norm_w), dev(np.ascontiguousarray(router, np.float32))
    out = empty_f32(T, H)
    sync(cuda)
    cuda.moe_block(xd.data_ptr(), wd.data_ptr(), rd.data_ptr(), L.ExpertPack(gq, pg.data_ptr(), sgs),
                   L.ExpertPack(gq, pu.data_ptr(), sus), L.ExpertPack(dq, pd.data_ptr(), sds), sh, out.data_ptr(), T,
                   H, I, E, top_k)
    cuda.synchronize()
    return host(out)


def check(oracle, got, x, norm_w, router, experts, shared, top_k):
    ref = oracle.moe_block(x, norm_w, (S.FP32, router), experts, shared, top_k=top_k)
    ref64 = oracle.moe_block(x, norm_w, (S.FP32, router), experts, shared, top_k=top_k, f64=True)
    for t in range(x.shape[0]):
        assert rel_err(got[t] - x[t], ref[t] - x[t]) <= TOL, t
        assert rel_err(got[t] - x[t], ref64[t] - x[t]) <= TOL, t
        assert rel_err(got[t], ref[t]) <= TOL, t


def block_case(seed, E, H, I, SI, T, gq=S.Q4_K, dq=S.Q6_K, shared_router=True):
    rng = np.random.Generator(np.random.PCG64(seed))
    gate, up, down = S.moe_weights(rng, E, gq, dq, H, I)
    router = (rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    shared = None
    if SI:
        sg, su = S.make_matrix(gq, SI, H, rng), S.make_matrix(gq, SI, H, rng)
        sd = S.make_matrix(dq, H, SI, rng)
        sr = (rng.standard_normal((1, H), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
        shared = ((gq, sg), (gq, su), (dq, sd), (S.FP32, sr) if shared_router else None)
    norm_w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    return x, norm_w, router, (gq, gate, up, dq, down), shared


def test_block_golden(cuda):
    """The fixture's inputs (regenerated from its seed) through the device
    block; outputs against qw6's own composition of the block."""
    from pathlib import Path

    from tests.golden.gen_golden import block_inputs
    g = np.load(Path(__file__).resolve().parent / "golden" / "moe_block.npz")
    b = block_inputs(int(g["seed"]))
    assert b["sha"] == str(g["sha"])
    K = b["dims"][4]
    for shared, want in ((b["shared"], g["out"]), (None, g["out_routed"])):
        got = run_block(cuda, b["x"], b["norm_w"], b["router"][1], b["experts"], shared, K)
        for t in range(b["x"].shape[0]):
            assert rel_err(got[t] - b["x"][t], want[t] - b["x"][t]) <= TOL, t


@pytest.mark.parametrize("T", [1, 3, 8])
@pytest.mark.parametrize("shared_kind", ["router", "no_router", "none"])
def test_block_vs_oracle(T, shared_kind, cuda, oracle):
    E, H, I, SI, K = 64, 2048, 512, 512, 8
    for seed in range(100, 140):
        x, nw, router, experts, shared = block_case(seed, E, H, I, SI if shared_kind != "none" else 0, T,
                                                    shared_router=shared_kind == "router")
        if routing_margin_ok(oracle, x, nw, router, K):
            break
    else:
        pytest.fail("no seed with a clear routing margin")
    got = run_block(cuda, x, nw, router, experts, shared, K)
    check(oracle, got, x, nw, router, experts, shared, K)


def test_block_iq_formats_256_experts(cuda, oracle):
    """256 experts with IQ2_XXS gate/up and down, one token (the decode case)."""
    for seed in range(200, 240):
        x, nw, router, experts, shared = block_case(seed, 256, 2048, 512, 512, 1, S.IQ2_XXS, S.IQ2_XXS)
        if routing_margin_ok(oracle, x, nw, router, 8):
            break
    got = run_block(cuda, x, nw, router, experts, shared, 8)
    check(oracle, got, x, nw, router, experts, shared, 8)
