"""GPU parity of the routing / combine / activation / argmax / fp32 kernels
(exact indices; fp32 values within the stated tolerances)."""
from pathlib import Path

import numpy as np
import pytest

from qw6_b200 import lib as L
from tests.conftest import rel_err, same_bits
from tests.gpu_util import dev, empty_f32, host, sync

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_route_golden_host_api():
    g = np.load(GOLDEN / "route.npz")
    for lg, idx, w in zip(g["logits"], g["idx"], g["w"]):
        gi, gw = L.moe_route_host(lg, 8)
        assert np.array_equal(gi.astype(np.int32), idx)
        ok = ~np.isnan(w)
        assert np.array_equal(np.isnan(gw), ~ok)
        assert np.allclose(gw[ok], w[ok], rtol=1e-5, atol=1e-7)


def test_route_batched_device_api(cuda, oracle, rng):
    T, E, K = 257, 256, 8
    lg = rng.standard_normal((T, E)).astype(np.float32)
    lg[::7, rng.integers(0, E, 5)] = 3.0  # ties
    ld = dev(lg)
    torch = pytest.importorskip("torch")
    idx = torch.empty(T * K, dtype=torch.int32, device="cuda")
    w = empty_f32(T * K)
    sync(cuda)
    cuda.moe_route(ld.data_ptr(), T, E, K, idx.data_ptr(), w.data_ptr())
    cuda.synchronize()
    gi, gw = host(idx).reshape(T, K), host(w).reshape(T, K)
    for t in range(T):
        oi, ow = oracle.moe_route(lg[t], K)
        assert np.array_equal(gi[t], oi)
        assert np.allclose(gw[t], ow, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("ne,k", [(256, 8), (128, 4), (64, 1), (8, 8), (37, 5)])
def test_route_shapes(ne, k, oracle, rng):
    lg = rng.standard_normal(ne).astype(np.float32)
    gi, gw = L.moe_route_host(lg, k)
    oi, ow = oracle.moe_route(lg, k)
    assert np.array_equal(gi.astype(np.int32), oi) and np.allclose(gw, ow, rtol=1e-5, atol=1e-7)


def test_route_rejects_bad_args():
    with pytest.raises(L.Qw6CudaError):
        L.moe_route_host(np.zeros(300, np.float32), 8)  # n_experts > 256
    with pytest.raises(L.Qw6CudaError):
        L.moe_route_host(np.zeros(64, np.float32), 9)  # top_k > 8


def test_gather_bitexact(oracle, rng):
    dim, k = 257, 8
    eo = rng.standard_normal((k, dim)).astype(np.float32)
    w = rng.random(k).astype(np.float32)
    sh = rng.standard_normal(dim).astype(np.float32)
    assert same_bits(L.moe_gather_host(eo, w, sh, 0.25, dim, k), oracle.moe_gather(eo, w, sh, 0.25, dim, k))
    assert same_bits(L.moe_gather_host(eo, w, None, 0.0, dim, k), oracle.moe_gather(eo, w, None, 0.0, dim, k))


def test_silu_mul(oracle, rng):
    g = (rng.standard_normal(4099) * 8).astype(np.float32)
    u = rng.standard_normal(4099).astype(np.float32)
    got = L.silu_mul_host(g, u)
    want = oracle.silu_mul(g, u)
    assert np.allclose(got, want, rtol=2e-6, atol=1e-30)


def test_argmax_golden():
    g = np.load(GOLDEN / "argmax.npz")
    for x, n, idx in zip(g["x"], g["n"], g["idx"]):
        i, v = L.argmax_host(x[:n])
        assert i == idx
        assert L.sampling_greedy_host(x[:n]) == idx


def test_argmax_large_ties(rng):
    x = rng.standard_normal(248320).astype(np.float32)
    x[[1000, 5, 200000]] = 7.5
    assert L.argmax_host(x) == (5, 7.5)


def test_matvec_f32(rng):
    rows, cols = 256, 2048
    w = rng.standard_normal((rows, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    y = L.matvec_f32_host(w, x, rows, cols)
    assert rel_err(y, w.astype(np.float64) @ x.astype(np.float64)) <= 1e-5
    w = rng.standard_normal((7, 19)).astype(np.float32)  # qw6_vk.c self-test shape
    x = rng.standard_normal(19).astype(np.float32)
    assert rel_err(L.matvec_f32_host(w, x, 7, 19), w.astype(np.float64) @ x) <= 1e-5
