"""GPU: one process driving two devices through two contexts.

Kernels that use more than 48 KB of dynamic shared memory need a function
attribute that CUDA keeps per device; the library sets it once on each device
it launches on.  This test runs those kernels (32-token matvec, the planned
decode MoE, the tensor-core prefill) on cuda:0 and then on cuda:1 from the
same process, checks cuda:0 against the oracle and cuda:1 bit for bit against
cuda:0.  Skipped with fewer than two GPUs."""
import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.conftest import rel_err, same_bits
from tests.gpu_util import dev, empty_f32, host, pack, sync

pytestmark = pytest.mark.gpu


def _need_two():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    return torch


def _matvec32(ctx, q, w, x, rows, cols):
    packed, _ = pack(ctx, q, w, rows, cols)
    xd = dev(x)
    y = empty_f32(x.shape[0], rows)
    sync(ctx)
    ctx.matvec(q, packed.data_ptr(), xd.data_ptr(), y.data_ptr(), rows, cols, x.shape[0])
    ctx.synchronize()
    return host(y)


def _moe(ctx, gate, up, down, logits, x, K):
    E, I, H = gate.shape[0], gate.shape[1], x.shape[1]
    pg, sg = pack(ctx, S.Q4_K, gate, I, H, E)
    pu, su = pack(ctx, S.Q4_K, up, I, H, E)
    pd, sd = pack(ctx, S.Q6_K, down, H, I, E)
    ld, xd = dev(logits), dev(x)
    out = empty_f32(x.shape[0], H)
    sync(ctx)
    ctx.moe_decode(L.ExpertPack(S.Q4_K, pg.data_ptr(), sg), L.ExpertPack(S.Q4_K, pu.data_ptr(), su),
                   L.ExpertPack(S.Q6_K, pd.data_ptr(), sd), ld.data_ptr(), xd.data_ptr(), out.data_ptr(),
                   x.shape[0], H, I, E, K)
    ctx.synchronize()
    return host(out)


def _prefill(ctx, gate, up, down, logits, xbits, K):
    E, I, H = gate.shape[0], gate.shape[1], xbits.shape[1]
    pg, sg = pack(ctx, S.Q4_K, gate, I, H, E)
    pu, su = pack(ctx, S.Q4_K, up, I, H, E)
    pd, sd = pack(ctx, S.Q6_K, down, H, I, E)
    ld, xd = dev(logits), dev(xbits.view(np.int16))
    out = empty_f32(xbits.shape[0], H)
    sync(ctx)
    ctx.moe_prefill(L.ExpertPack(S.Q4_K, pg.data_ptr(), sg), L.ExpertPack(S.Q4_K, pu.data_ptr(), su),
                    L.ExpertPack(S.Q6_K, pd.data_ptr(), sd), ld.data_ptr(), xd.data_ptr(), out.data_ptr(),
                    xbits.shape[0], H, I, E, K)
    ctx.check_device_errors()
    return host(out)


def test_large_smem_kernels_on_both_devices(oracle):
    torch = _need_two()
    rng = np.random.Generator(np.random.PCG64(2024))
    q, rows, cols = S.IQ2_S, 2048, 4096
    w = S.make_matrix(q, rows, cols, rng)
    xm = rng.standard_normal((32, cols), dtype=np.float32)
    E, H, I, K = 32, 2048, 512, 8
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    lg = rng.standard_normal((12, E), dtype=np.float32)
    xd = rng.standard_normal((12, H), dtype=np.float32)
    T = 200
    lp = rng.standard_normal((T, E), dtype=np.float32)
    xb = S.bf16_round(rng.standard_normal((T, H), dtype=np.float32))

    results = []
    for d in (0, 1):
        with torch.cuda.device(d):
            ctx = L.Context(d)
            try:
                results.append((_matvec32(ctx, q, w, xm, rows, cols), _moe(ctx, gate, up, down, lg, xd, K),
                                _prefill(ctx, gate, up, down, lp, xb, K)))
            finally:
                ctx.close()

    (mv0, moe0, pf0), (mv1, moe1, pf1) = results
    ref = oracle.matvec(q, w, xm, rows, cols).reshape(32, rows)
    assert max(rel_err(mv0[t], ref[t]) for t in range(32)) <= 1e-3
    ref_moe, _, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, lg, xd, top_k=K)
    assert max(rel_err(moe0[t], ref_moe[t]) for t in range(12)) <= 1e-3
    toks = list(range(0, T, 10))
    ref_pf, _, _ = oracle.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, lp[toks], S.bf16_to_f32(xb)[toks], top_k=K)
    assert max(rel_err(pf0[t], ref_pf[i]) for i, t in enumerate(toks)) <= 2e-2
    # the second device runs the same kernels on the same inputs
    assert same_bits(mv1, mv0)
    assert same_bits(moe1, moe0)
    assert same_bits(pf1, pf0)
