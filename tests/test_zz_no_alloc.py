"""GPU: the allocation-free MoE entry point (qw6cu_moe_decode_noalloc).

Some callers cannot call cudaMalloc at the point where they run the MoE layer:
a runtime or serving process that hands out all device memory from its own
pool, or one whose device-memory footprint must stay fixed after start-up (an
allocation there can fail, or stall on device-wide synchronisation, at a
point where neither is acceptable). For them the library keeps a fixed 1 MiB
scratch array in device memory and this entry point works only out of that
array, plus the caller's own inputs and outputs.

The test checks it through the C ABI against qw6cu_moe_decode (the entry point
that uses the context's workspace) on two calls in a row, which also covers
reuse of the shared scratch.  It is collected last (file name) and sets up
everything it needs, so it passes alone in a fresh process and after the rest.
"""
import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.conftest import rel_err
from tests.gpu_util import dev, empty_f32, host, pack, sync

pytestmark = pytest.mark.gpu
TOL = 1e-3  # same bar as the other MoE parity tests (max rel err)


def _packs(cuda, rng, E, H, I):
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    pg, sg = pack(cuda, S.Q4_K, gate, I, H, E)
    pu, su = pack(cuda, S.Q4_K, up, I, H, E)
    pd, sd = pack(cuda, S.Q6_K, down, H, I, E)
    keep = (pg, pu, pd)
    return keep, (L.ExpertPack(S.Q4_K, pg.data_ptr(), sg), L.ExpertPack(S.Q4_K, pu.data_ptr(), su),
                  L.ExpertPack(S.Q6_K, pd.data_ptr(), sd))


@pytest.mark.parametrize("ntok,E", [(1, 32), (4, 32), (8, 32), (12, 256)])
def test_noalloc_matches_workspace_entry_point(ntok, E):
    """ntok 1 and 4 take the two-kernel small-batch path, 8 and 12 the planned
    path; 12 tokens over 256 experts is the largest batch whose workspace
    fits the fixed scratch."""
    torch = pytest.importorskip("torch")
    rng = np.random.Generator(np.random.PCG64(99 + ntok))
    H, I, K = 2048, 512, 8
    assert L.Context.moe_workspace_bytes(ntok, H, I, E, K) <= 1 << 20
    ctx = L.Context(0)
    keep, (g, u, d) = _packs(ctx, rng, E, H, I)
    logits = dev(rng.standard_normal((ntok, E), dtype=np.float32))
    x = dev(rng.standard_normal((ntok, H), dtype=np.float32))
    ref = empty_f32(ntok, H)
    sync(ctx)
    ctx.moe_decode(g, u, d, logits.data_ptr(), x.data_ptr(), ref.data_ptr(), ntok, H, I, E, K)
    ctx.synchronize()
    want = host(ref)
    for _ in range(2):  # two calls in a row share (and reuse) the fixed scratch
        out = empty_f32(ntok, H)
        out.fill_(float("nan"))
        torch.cuda.synchronize()
        L.moe_decode_noalloc(g, u, d, logits.data_ptr(), x.data_ptr(), out.data_ptr(), ntok, H, I, E, K, stream=0)
        got = host(out)
        for t in range(ntok):
            assert rel_err(got[t], want[t]) <= TOL, t
    del keep
    ctx.close()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """64 tokens need more than the 1 MiB scratch: a clear error, no launch."""
    with pytest.raises(L.Qw6CudaError, match="fixed scratch"):
        L.moe_decode_noalloc(L.ExpertPack(S.Q4_K, 256, 0), L.ExpertPack(S.Q4_K, 256, 0),
                             L.ExpertPack(S.Q6_K, 256, 0), 256, 256, 256, 64, 2048, 512, 256, 8, stream=0)


def test_noalloc_on_two_devices():
    """Each device has its own copy of the fixed scratch: the entry point runs
    on whichever device is current, and its kernels' per-device set-up is done
    on first use there.  Skipped with fewer than two GPUs."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ntok, E, H, I, K = 8, 32, 2048, 512, 8
    for d in (0, 1):
        with torch.cuda.device(d):
            rng = np.random.Generator(np.random.PCG64(7))
            ctx = L.Context(d)
            keep, (g, u, dn) = _packs(ctx, rng, E, H, I)
            logits = dev(rng.standard_normal((ntok, E), dtype=np.float32))
            x = dev(rng.standard_normal((ntok, H), dtype=np.float32))
            ref = empty_f32(ntok, H)
            sync(ctx)
            ctx.moe_decode(g, u, dn, logits.data_ptr(), x.data_ptr(), ref.data_ptr(), ntok, H, I, E, K)
            ctx.synchronize()
            want = host(ref)
            out = empty_f32(ntok, H)
            out.fill_(float("nan"))
            torch.cuda.synchronize()
            L.moe_decode_noalloc(g, u, dn, logits.data_ptr(), x.data_ptr(), out.data_ptr(), ntok, H, I, E, K,
                                 stream=0)
            got = host(out)
            for t in range(ntok):
                assert rel_err(got[t], want[t]) <= TOL, (d, t)
            del keep
            ctx.close()
