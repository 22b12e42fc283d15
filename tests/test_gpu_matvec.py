"""GPU parity: dequantization (bit-exact) and fused dequant-matvec (max
relative error <= 1e-3) against the CPU oracle and the
golden fixtures made by qw6's own code.  All calls go through the C ABI."""
from pathlib import Path

import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.conftest import rel_err, same_bits
from tests.gpu_util import dev, empty_f32, host, pack, sync

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 1e-3  # max|y - y_ref| / max|y_ref|
SHAPES = [(1, 256), (7, 512), (16, 2048), (33, 2048), (512, 2048), (2048, 512), (100, 4096)]


def gpu_dequant(cuda, q, w, rows, cols):
    raw = dev(w.reshape(-1).view(np.uint8))
    out = empty_f32(rows, cols)
    sync(cuda)
    cuda.dequantize(q, raw.data_ptr(), out.data_ptr(), rows, cols)
    cuda.synchronize()
    return host(out)


def gpu_matvec(cuda, q, w, x, rows, cols):
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    ntok = x.shape[0]
    pk, _ = pack(cuda, q, w, rows, cols)
    xd = dev(x)
    y = empty_f32(ntok, rows)
    sync(cuda)
    cuda.matvec(q, pk.data_ptr(), xd.data_ptr(), y.data_ptr(), rows, cols, ntok)
    cuda.synchronize()
    return host(y)


@pytest.mark.parametrize("q", S.BLOCK_QUANTS)
def test_dequant_bitexact_random(q, cuda, oracle, rng):
    for rows, cols in [(7, 512), (64, 2048)]:
        w = S.make_matrix(q, rows, cols, rng)
        assert same_bits(gpu_dequant(cuda, q, w, rows, cols), oracle.dequantize(q, w, rows, cols))


@pytest.mark.parametrize("name", [S.QUANT_NAMES[q] for q in S.BLOCK_QUANTS])
def test_dequant_bitexact_golden(name, cuda):
    g = np.load(GOLDEN / f"matvec_{name}.npz")
    q, rows, cols = int(g["quant"]), int(g["rows"]), int(g["cols"])
    assert same_bits(gpu_dequant(cuda, q, g["w"], rows, cols), g["deq"])
    ns = g["w_special"].shape[0]
    assert same_bits(gpu_dequant(cuda, q, g["w_special"], ns, cols), g["deq_special"])


@pytest.mark.parametrize("q", S.BLOCK_QUANTS)
def test_matvec_vs_oracle(q, cuda, oracle, rng):
    for rows, cols in SHAPES:
        w = S.make_matrix(q, rows, cols, rng)
        x = rng.standard_normal(cols, dtype=np.float32)
        y = gpu_matvec(cuda, q, w, x, rows, cols)[0]
        assert rel_err(y, oracle.matvec(q, w, x, rows, cols)) <= TOL, (rows, cols)
        assert rel_err(y, oracle.matvec_f64(q, w, x, rows, cols)) <= TOL


@pytest.mark.parametrize("q", S.BLOCK_QUANTS)
@pytest.mark.parametrize("ntok", [2, 3, 4, 5, 8, 13, 32])
def test_matvec_multi_token(q, ntok, cuda, oracle, rng):
    rows, cols = 48, 2048
    w = S.make_matrix(q, rows, cols, rng)
    x = rng.standard_normal((ntok, cols), dtype=np.float32)
    y = gpu_matvec(cuda, q, w, x, rows, cols)
    ref = oracle.matvec(q, w, x, rows, cols).reshape(ntok, rows)
    for t in range(ntok):
        assert rel_err(y[t], ref[t]) <= TOL, t


@pytest.mark.parametrize("ntok", [20, 32])
def test_matvec_wide_batch(ntok, cuda, oracle, rng):
    """Config 4's IQ2_S shape [2048 x 4096] at batch 32: the 32-token
    activation stage of 4096 columns exceeds shared memory, so the launch is
    split into 16-token chunks."""
    q, rows, cols = S.IQ2_S, 2048, 4096
    w = S.make_matrix(q, rows, cols, rng)
    x = rng.standard_normal((ntok, cols), dtype=np.float32)
    y = gpu_matvec(cuda, q, w, x, rows, cols)
    ref = oracle.matvec(q, w, x, rows, cols).reshape(ntok, rows)
    for t in range(ntok):
        assert rel_err(y[t], ref[t]) <= TOL, t


def _halves(rng, q, rows, cols):
    """FP16 / BF16 weight rows with special values mixed in: +-0, subnormals,
    +-inf, NaN (for FP16 the exact widening of qw6_fp16_to_f32 is checked)."""
    if q == S.FP16:
        h = rng.standard_normal((rows, cols)).astype(np.float16).view(np.uint16)
        special = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x8001, 0x7C00, 0xFC00, 0x7E00, 0x7BFF], np.uint16)
    else:
        h = S.bf16_round(rng.standard_normal((rows, cols)).astype(np.float32))
        special = np.array([0x0000, 0x8000, 0x0001, 0x007F, 0x7F80, 0xFF80, 0x7FC0, 0x7F7F], np.uint16)
    h.reshape(-1)[: special.size] = special
    return h.view(np.uint8).reshape(rows, cols * 2)


@pytest.mark.parametrize("q", [S.FP16, S.BF16])
def test_dequant16_bitexact(q, cuda, oracle, rng):
    """FP16 / BF16 rows (qw6.c:1686-1692): the exact widening, bit for bit
    (NaN positions only for NaN)."""
    rows, cols = 9, 1000
    w = _halves(rng, q, rows, cols)
    assert same_bits(gpu_dequant(cuda, q, w, rows, cols), oracle.dequantize(q, w, rows, cols))


@pytest.mark.parametrize("q", [S.FP16, S.BF16])
@pytest.mark.parametrize("ntok", [1, 3, 8, 32])
def test_matvec16_vs_oracle(q, ntok, cuda, oracle, rng):
    """16-bit weight matvec (row-major, no repacking), 1-32 tokens, against the
    oracle's dequant-then-dot (qw6_tensor_matvec order) and its float64 form."""
    rows, cols = 333, 1000
    w = _halves(rng, q, rows, cols)
    w.view(np.uint16).reshape(-1)[:16] = 0  # keep the specials out of the dot
    x = rng.standard_normal((ntok, cols), dtype=np.float32)
    y = gpu_matvec(cuda, q, w, x, rows, cols)
    ref = oracle.matvec(q, w, x, rows, cols).reshape(ntok, rows)
    for t in range(ntok):
        assert rel_err(y[t], ref[t]) <= TOL, t
        assert rel_err(y[t], oracle.matvec_f64(q, w, x[t], rows, cols)) <= TOL, t


def test_matvec_heavy_tailed_activations(cuda, oracle, rng):
    """Per-256-block activation scaling copes with outliers (like silu*up)."""
    q, rows, cols = S.Q6_K, 256, 512
    w = S.make_matrix(q, rows, cols, rng)
    x = (rng.standard_normal(cols) ** 3 * 1e4).astype(np.float32)
    x[::97] *= 50
    y = gpu_matvec(cuda, q, w, x, rows, cols)[0]
    assert rel_err(y, oracle.matvec_f64(q, w, x, rows, cols)) <= TOL


@pytest.mark.parametrize("name", [S.QUANT_NAMES[q] for q in S.BLOCK_QUANTS])
def test_host_api_golden(name):
    """qw6_vk_matmul_<fmt>_host with host buffers, against qw6's output."""
    g = np.load(GOLDEN / f"matvec_{name}.npz")
    q, rows, cols = int(g["quant"]), int(g["rows"]), int(g["cols"])
    y = L.matmul_host(q, g["w"], g["x"], rows, cols)
    assert rel_err(y, g["y"]) <= TOL


@pytest.mark.parametrize("q", S.BLOCK_QUANTS)
def test_host_api_config_shapes(q, oracle, rng):
    shape = {S.Q4_K: (512, 2048), S.Q5_K: (4096, 2048), S.Q6_K: (2048, 512), S.IQ2_XXS: (512, 2048),
             S.IQ2_S: (2048, 4096), S.IQ3_S: (2048, 2048)}[q]
    rows, cols = shape
    w = S.make_matrix(q, rows, cols, rng)
    x = rng.standard_normal(cols, dtype=np.float32)
    assert rel_err(L.matmul_host(q, w, x, rows, cols), oracle.matvec(q, w, x, rows, cols)) <= TOL


def test_host_api_errors():
    w = np.zeros(144, np.uint8)
    x = np.zeros(256, np.float32)
    with pytest.raises(L.Qw6CudaError):
        L.matmul_host(S.Q4_K, w, x, 1, 100)  # cols not a multiple of 256
    with pytest.raises(L.Qw6CudaError):
        L.matmul_host(S.Q4_K, w, x, 0, 256)  # no rows


def test_selftest_kats():
    """qw6_vk_selftest: the closed-form KATs of qw6's Vulkan self-test."""
    assert L.selftest() == 0


@pytest.mark.parametrize("q,rows,cols", [(S.Q5_K, 4096, 2048), (S.Q4_K, 512, 2048), (S.IQ3_S, 2048, 2048)])
@pytest.mark.parametrize("ntok", [6, 20, 32])
def test_matvec_token_chunks(q, rows, cols, ntok, cuda, oracle, rng):
    """Config 0 / 4 shapes at batches above 4, which run as token chunks side
    by side (4 tokens a chunk, or 16 for mid-sized K-format matrices)."""
    w = S.make_matrix(q, rows, cols, rng)
    x = rng.standard_normal((ntok, cols), dtype=np.float32)
    y = gpu_matvec(cuda, q, w, x, rows, cols)
    ref = oracle.matvec(q, w, x, rows, cols).reshape(ntok, rows)
    for t in range(ntok):
        assert rel_err(y[t], ref[t]) <= TOL, t
