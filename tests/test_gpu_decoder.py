"""GPU: the decode-step executor (qw6cu_decoder_*, and qw6's own pipeline
entry points qw6_vk_pipe_* on top of it) against qw6's forward pass
(qw6_forward_token, qw6.c:2426-2500): the oracle's restatement for small
models over 40 positions (two attention chunks), and qw6 itself -- its
session driving this library through qw6_vk_pipe_forward against its own CPU
path -- for the full 40-layer stack.  Tolerance on the logits of every
position: max relative error 1e-3 (fp32 path; the matvecs quantize
activations to 15-bit fixed point per 256-block, sums run in another order).
The greedy pick must be the argmax of the logits returned with it, and
qw6's pick unless the top two logits are within that tolerance."""
import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _close_pick(pick, ref_row):
    top = np.sort(ref_row)[-2:]
    return pick == int(np.argmax(ref_row)) or (top[1] - top[0]) <= TOL * np.abs(ref_row).max()


@pytest.fixture(scope="module")
def small():
    return S.fwd_model(seed=21, n_layers=4, vocab=4096, embd_rows=4096, attn_period=4, expert_period=4)


@pytest.fixture(scope="module")
def small_ref(small, oracle):
    tokens = [int(t) for t in np.random.Generator(np.random.PCG64(3)).integers(0, 4096, 40)]
    return tokens, oracle.forward(small, tokens)


def test_decoder_matches_oracle(cuda, small, small_ref):
    tokens, want = small_ref
    dec = L.Decoder(cuda, small, max_ctx=64)
    try:
        for pos, tok in enumerate(tokens):
            got, pick = dec.forward(tok, pos)
            assert rel_err(got, want[pos]) <= TOL, pos
            assert pick == int(np.argmax(got))
            assert _close_pick(pick, want[pos]), pos
    finally:
        dec.close()


def test_decoder_generate_and_reset(cuda, small):
    """generate() chains greedy steps on the device: the same ids as feeding
    each step's pick back through forward(); reset() clears the state."""
    dec = L.Decoder(cuda, small, max_ctx=32)
    try:
        gen = dec.generate(17, 0, 6)
        dec.reset()
        tok, picks, first = 17, [], None
        for pos in range(6):
            logits, tok = dec.forward(tok, pos)
            picks.append(tok)
            if pos == 0:
                first = logits
        assert list(gen) == picks
        dec.reset()
        again, _ = dec.forward(17, 0)
        assert np.array_equal(again.view(np.uint32), first.view(np.uint32))
    finally:
        dec.close()


def test_decoder_without_shared_expert(cuda, oracle):
    m = S.fwd_model(seed=22, n_layers=4, vocab=1024, embd_rows=128, attn_period=4, expert_period=4, shared=False)
    tokens = [3, 99, 42]
    want = oracle.forward(m, tokens)
    dec = L.Decoder(cuda, m, max_ctx=8)
    try:
        for pos, tok in enumerate(tokens):
            got, _ = dec.forward(tok, pos)
            assert rel_err(got, want[pos]) <= TOL, pos
    finally:
        dec.close()


def test_decoder_other_formats(cuda, oracle):
    """Q4_K attention/shared weights, IQ3_S experts, and FP16 alpha/beta."""
    m = S.fwd_model(seed=23, n_layers=4, vocab=1024, embd_rows=128, attn_period=4, expert_period=4,
                    weight_quant=S.Q4_K, expert_quant=S.IQ3_S)
    rng = np.random.Generator(np.random.PCG64(5))
    swap = {}
    for i, (f, l, q, r, c, arr, st) in enumerate(m.tensors):
        if f in (S.F_DN_ALPHA, S.F_DN_BETA):
            h = (rng.standard_normal((r, c)) * 0.02).astype(np.float16).view(np.uint8)
            swap[i] = (f, l, S.FP16, r, c, h, 0)
    for i, t in swap.items():
        m.tensors[i] = t
    tokens = [1, 2, 3]
    want = oracle.forward(m, tokens)
    dec = L.Decoder(cuda, m, max_ctx=8)
    try:
        for pos, tok in enumerate(tokens):
            got, _ = dec.forward(tok, pos)
            assert rel_err(got, want[pos]) <= TOL, pos
    finally:
        dec.close()


def test_decoder_reports_non_finite_and_bad_input(cuda, small):
    dec = L.Decoder(cuda, small, max_ctx=4)
    try:
        with pytest.raises(L.Qw6CudaError):
            dec.forward(1, 4)  # past max_ctx
        with pytest.raises(L.Qw6CudaError):
            dec.forward(4096, 0)  # past the embedding rows
    finally:
        dec.close()
    bad = S.FwdModel(small.n_layers, small.vocab, small.embd_rows)
    for t in small.tensors:
        f, l, q, r, c, arr, st = t
        if f == S.F_NORM and l == 1:
            arr = arr.copy()
            arr[0, 5] = np.inf
        bad.add(f, l, q, r, c, arr, st)
    dec = L.Decoder(cuda, bad, max_ctx=4)
    try:
        with pytest.raises(L.Qw6CudaError, match="non-finite"):
            dec.forward(1, 0)
    finally:
        dec.close()
    short = S.FwdModel(small.n_layers, small.vocab, small.embd_rows)
    for t in small.tensors:
        if not (t[0] == S.F_DN_NORM and t[1] == 2):
            short.add(*t)
    with pytest.raises(L.Qw6CudaError, match="lacks tensor"):
        L.Decoder(cuda, short, max_ctx=4)


def test_qw6_pipeline_drives_the_decoder():
    """qw6's own session (qw6.c built with QW6_VULKAN against this library,
    oracle/_ref/libqw6vk.so): qw6_prefill through qw6_vk_pipe_forward against
    the same library's CPU forward, 40 layers, three positions; and
    qw6_vk_pipe_forward_greedy's picks.  The synthetic model writes updates of
    0.1 of the residual stream per layer (synth.fwd_model's out_scale): with
    O(1) updates a random 40-layer stack amplifies relative differences of
    1e-5 (the activation quantization of the matvecs) beyond 1e-3 in qw6's
    own fp32 forward pass, and flips expert choices."""
    from oracle.oracle import VkReference
    if not VkReference.available():
        pytest.skip("oracle/_ref/libqw6vk.so not built (reference tree absent when building)")
    vk = VkReference()
    m = S.fwd_model(seed=24, n_layers=40, vocab=4096, embd_rows=1024)
    tokens = [11, 500, 1023]
    want = vk.forward(m, tokens, use_pipe=False)
    got = vk.forward(m, tokens, use_pipe=True)
    for pos in range(len(tokens)):
        assert rel_err(got[pos], want[pos]) <= TOL, pos
    picks, logits = vk.pipe_greedy(m, tokens)
    for pos in range(len(tokens)):
        assert rel_err(logits[pos], want[pos]) <= TOL, pos
        assert int(picks[pos]) == int(np.argmax(logits[pos]))
        assert _close_pick(int(picks[pos]), want[pos]), pos
