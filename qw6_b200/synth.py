"""Seeded synthetic GGUF super-blocks and activations.

No GGUF model file is used anywhere: every weight matrix is generated here
from a numpy PCG64 stream, with the value distributions of the benchmark
configurations (fp16 scales drawn as |N(0,1)| x 0.01 for the K formats and
x 0.02 for the IQ formats, everything else uniform random bytes, Q6_K
scales uniform int8 in [-32, 31]).  fp16 fields use round-to-nearest-even
(np.float16).  The same bytes feed the CUDA library and the CPU oracle.
"""
from __future__ import annotations

import numpy as np

# qw6_quant_t codes (qw6.h:77-92)
FP32, FP16, BF16, Q8_0, Q4_K, Q4_K_S, Q5_K, Q6_K = 0, 1, 2, 3, 4, 5, 6, 7
IQ3_S, IQ2_S, IQ2_M, IQ2_XXS = 9, 11, 12, 13

BLOCK_BYTES = {Q4_K: 144, Q4_K_S: 144, Q5_K: 176, Q6_K: 210,
               IQ2_XXS: 66, IQ2_S: 82, IQ3_S: 110}
QUANT_NAMES = {Q4_K: "q4k", Q5_K: "q5k", Q6_K: "q6k", IQ2_XXS: "iq2xxs",
               IQ2_S: "iq2s", IQ3_S: "iq3s"}
BLOCK_QUANTS = (Q4_K, Q5_K, Q6_K, IQ2_XXS, IQ2_S, IQ3_S)

# hidden 2048, 256 experts, top-8, expert intermediate 512 (qw6.h:24-73)
HIDDEN, N_EXPERTS, TOP_K, INTER, VOCAB = 2048, 256, 8, 512, 248320


def row_bytes(quant: int, cols: int) -> int:
    if quant == FP32:
        return 4 * cols
    if quant in (FP16, BF16):
        return 2 * cols
    assert cols % 256 == 0
    return cols // 256 * BLOCK_BYTES[quant]


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(v.astype(np.float16)).view(np.uint8).reshape(-1, 2)


def make_blocks(quant: int, nblocks: int, rng: np.random.Generator,
                dscale: float | None = None) -> np.ndarray:
    """nblocks super-blocks of `quant` as a uint8 array [nblocks, block]."""
    bb = BLOCK_BYTES[quant]
    b = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    if quant in (Q4_K, Q4_K_S, Q5_K):
        s = 0.01 if dscale is None else dscale
        b[:, 0:2] = _f16_bytes(np.abs(rng.standard_normal(nblocks)) * s)
        b[:, 2:4] = _f16_bytes(np.abs(rng.standard_normal(nblocks)) * s)
    elif quant == Q6_K:
        s = 0.01 if dscale is None else dscale
        b[:, 192:208] = rng.integers(-32, 32, size=(nblocks, 16), dtype=np.int8).view(np.uint8)
        b[:, 208:210] = _f16_bytes(np.abs(rng.standard_normal(nblocks)) * s)
    else:  # IQ2_XXS, IQ2_S, IQ3_S: d first, the rest random
        s = 0.02 if dscale is None else dscale
        b[:, 0:2] = _f16_bytes(np.abs(rng.standard_normal(nblocks)) * s)
    return b


def make_matrix(quant: int, rows: int, cols: int, rng: np.random.Generator,
                dscale: float | None = None) -> np.ndarray:
    """Row-major [rows, row_bytes] uint8 matrix of random super-blocks."""
    if quant == FP32:
        return rng.standard_normal((rows, cols), dtype=np.float32).view(np.uint8)
    nb = cols // 256
    return make_blocks(quant, rows * nb, rng, dscale).reshape(rows, nb * BLOCK_BYTES[quant])


def make_expert_pack(quant: int, n_experts: int, rows: int, cols: int,
                     rng: np.random.Generator) -> np.ndarray:
    """GGUF-style expert pack: expert e at e*rows*row_bytes (qw6.c:592-594)."""
    return make_matrix(quant, n_experts * rows, cols, rng).reshape(n_experts, rows, -1)


# ---- benchmark configurations (seed = config index) ----

def config0(seed: int = 0):
    """Q4_K matvec 512x2048, x fp32[2048] ~ N(0,1)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    w = make_matrix(Q4_K, 512, 2048, rng)
    x = rng.standard_normal(2048, dtype=np.float32)
    return w, x


def moe_weights(rng, n_experts=N_EXPERTS, gate_q=Q4_K, down_q=Q6_K,
                hidden=HIDDEN, inter=INTER):
    gate = make_expert_pack(gate_q, n_experts, inter, hidden, rng)
    up = make_expert_pack(gate_q, n_experts, inter, hidden, rng)
    down = make_expert_pack(down_q, n_experts, hidden, inter, rng)
    return gate, up, down


def config1(seed: int = 1, n_experts: int = N_EXPERTS):
    """MoE decode b=1: logits fp32[256] ~ N(0,1), Q4_K gate/up, Q6_K down."""
    rng = np.random.Generator(np.random.PCG64(seed))
    gate, up, down = moe_weights(rng, n_experts)
    logits = rng.standard_normal((1, n_experts), dtype=np.float32)
    x = rng.standard_normal((1, HIDDEN), dtype=np.float32)
    return gate, up, down, logits, x


def config2(seed: int = 2, ntok: int = 64, n_experts: int = N_EXPERTS):
    """Batched-decode MoE, IQ2_XXS experts, 64 tokens."""
    rng = np.random.Generator(np.random.PCG64(seed))
    gate, up, down = moe_weights(rng, n_experts, IQ2_XXS, IQ2_XXS)
    logits = rng.standard_normal((ntok, n_experts), dtype=np.float32)
    x = rng.standard_normal((ntok, HIDDEN), dtype=np.float32)
    return gate, up, down, logits, x


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round-to-nearest-even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def config3(seed: int = 3, ntok: int = 4096, n_experts: int = N_EXPERTS, with_bias: bool = False):
    """Prefill MoE: logits N(0,1) + per-expert bias N(0,0.5); X bf16.
    with_bias: also return the router bias (the model's share of the
    logits), from which `router_sample` draws independent token batches."""
    rng = np.random.Generator(np.random.PCG64(seed))
    gate, up, down = moe_weights(rng, n_experts)
    bias = (rng.standard_normal(n_experts) * 0.5).astype(np.float32)
    logits = rng.standard_normal((ntok, n_experts), dtype=np.float32) + bias[None, :]
    x = bf16_round(rng.standard_normal((ntok, HIDDEN), dtype=np.float32))
    if with_bias:
        return gate, up, down, logits.astype(np.float32), x, bias
    return gate, up, down, logits.astype(np.float32), x


def router_sample(bias: np.ndarray, ntok: int, seed: int) -> np.ndarray:
    """Router logits of another batch of the same model as config3: fresh
    N(0,1) token noise plus the given per-expert bias."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.standard_normal((ntok, bias.shape[0]), dtype=np.float32) + bias[None, :]).astype(np.float32)


def config4(seed: int = 4, batch: int = 1, vocab: int = VOCAB):
    """Mixed projections + Q6_K LM head."""
    rng = np.random.Generator(np.random.PCG64(seed))
    mats = {
        "q5k": (Q5_K, make_matrix(Q5_K, 4096, 2048, rng), 4096, 2048),
        "iq2s": (IQ2_S, make_matrix(IQ2_S, 2048, 4096, rng), 2048, 4096),
        "iq3s": (IQ3_S, make_matrix(IQ3_S, 2048, 2048, rng), 2048, 2048),
    }
    head = make_matrix(Q6_K, vocab, 2048, rng)
    xs = {k: rng.standard_normal((batch, c), dtype=np.float32) for k, (_, _, _, c) in mats.items()}
    h = rng.standard_normal((batch, 2048), dtype=np.float32)
    return mats, xs, head, h


# ---- a whole qw6 model for the decode-step executor ----
# Roles of the tensors (qw6_model_t's fields, qw6.h:126-170; the values of
# include/qw6_cuda.h's QW6CU_F_*).
(F_NORM, F_POST_NORM, F_ATTN_Q, F_ATTN_K, F_ATTN_V, F_ATTN_O, F_ATTN_Q_NORM, F_ATTN_K_NORM, F_ATTN_GATE,
 F_CONV1D, F_DN_OUT, F_DN_NORM, F_DN_ALPHA, F_DN_BETA, F_DN_DT, F_DN_A, F_MOE_ROUTER, F_SHARED_ROUTER,
 F_SHARED_GATE, F_SHARED_UP, F_SHARED_DOWN, F_EXPERT_GATE, F_EXPERT_UP, F_EXPERT_DOWN) = range(24)
F_TOK_EMBD, F_OUTPUT, F_OUTPUT_NORM = 100, 101, 102
N_LAYERS = 40


def is_full_attn(layer: int) -> bool:
    """qw6_layer_type (qw6.h:320-324): every 4th layer is full attention."""
    return layer % 4 == 3


class FwdModel:
    """Tensors of a qw6 model: (field, layer, quant, rows, cols, array, stride)
    with raw GGUF rows in `array` (uint8, or float32 for FP32 tensors); the
    expert packs hold all 256 experts, `stride` bytes apart."""

    def __init__(self, n_layers: int, vocab: int, embd_rows: int):
        self.n_layers, self.vocab, self.embd_rows = n_layers, vocab, embd_rows
        self.tensors: list[tuple[int, int, int, int, int, np.ndarray, int]] = []

    def add(self, field, layer, quant, rows, cols, arr, stride=0):
        self.tensors.append((field, layer, quant, rows, cols, np.ascontiguousarray(arr), stride))

    def nbytes(self) -> int:
        seen, n = set(), 0
        for t in self.tensors:
            if id(t[5]) not in seen:
                seen.add(id(t[5]))
                n += t[5].nbytes
        return n


def fwd_model(seed: int = 5, n_layers: int = N_LAYERS, vocab: int = 8192, embd_rows: int = 4096,
              attn_period: int = 8, expert_period: int = 2, expert_quant: int = IQ2_XXS,
              weight_quant: int = Q6_K, shared: bool = True, out_scale: float = 0.1) -> FwdModel:
    """A seeded qw6 model with qw6's dimensions (qw6.h:24-55) and the quant mix
    of its model card's primary plan: IQ2 experts, Q6_K attention, shared
    expert, embeddings and LM head, FP32 norms, router and conv weights.
    Scales keep activations O(1); the matrices that write into the residual
    stream (attention / DeltaNet output, expert and shared-expert down) are
    scaled by out_scale, so that every layer adds a small update to it as in
    a trained model: a random model with O(1) updates amplifies rounding
    differences about 100x over 40 layers.  Layer l reuses the
    weights of layer l % attn_period (attention, norms, router, shared
    expert) and l % expert_period (experts), so that 40 layers stay small
    on the host; both periods must be multiples of 4 or >= n_layers for the
    attention kind to match (experts: any)."""
    assert attn_period % 4 == 0 or attn_period >= n_layers
    rng = np.random.Generator(np.random.PCG64(seed))
    m = FwdModel(n_layers, vocab, embd_rows)
    ws = 1e-4 if weight_quant in (Q4_K, Q5_K, Q6_K) else 5e-4
    es = 5e-4 if expert_quant in (IQ2_XXS, IQ2_S, IQ3_S) else 1e-4

    def mat(q, rows, cols, s):
        if q == FP32:
            return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(s * 200)).astype(np.float32)
        if q in (FP16, BF16):
            v = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(s * 200)
            return (v.astype(np.float16).view(np.uint16) if q == FP16 else bf16_round(v)).view(np.uint8)
        return make_matrix(q, rows, cols, rng, s)

    def vec(n, base=1.0, s=0.1):
        return (base + s * rng.standard_normal((1, n))).astype(np.float32)

    sets: dict[int, list] = {}
    esets: dict[int, tuple] = {}
    for l in range(n_layers):
        a = l % attn_period if attn_period < n_layers else l
        if a not in sets:
            t = [(F_NORM, FP32, 1, HIDDEN, vec(HIDDEN)), (F_POST_NORM, FP32, 1, HIDDEN, vec(HIDDEN))]
            if is_full_attn(l):
                t += [(F_ATTN_Q, weight_quant, 8192, HIDDEN, mat(weight_quant, 8192, HIDDEN, ws)),
                      (F_ATTN_K, weight_quant, 512, HIDDEN, mat(weight_quant, 512, HIDDEN, ws)),
                      (F_ATTN_V, weight_quant, 512, HIDDEN, mat(weight_quant, 512, HIDDEN, ws)),
                      (F_ATTN_O, weight_quant, HIDDEN, 4096, mat(weight_quant, HIDDEN, 4096, ws * out_scale)),
                      (F_ATTN_Q_NORM, FP32, 1, 256, vec(256)), (F_ATTN_K_NORM, FP32, 1, 256, vec(256))]
            else:
                t += [(F_ATTN_Q, weight_quant, 8192, HIDDEN, mat(weight_quant, 8192, HIDDEN, ws)),
                      (F_ATTN_GATE, weight_quant, 4096, HIDDEN, mat(weight_quant, 4096, HIDDEN, ws)),
                      (F_DN_BETA, weight_quant, 32, HIDDEN, mat(weight_quant, 32, HIDDEN, ws)),
                      (F_DN_ALPHA, weight_quant, 32, HIDDEN, mat(weight_quant, 32, HIDDEN, ws)),
                      (F_DN_OUT, weight_quant, HIDDEN, 4096, mat(weight_quant, HIDDEN, 4096, ws * out_scale)),
                      (F_CONV1D, FP32, 8192, 4, (rng.standard_normal((8192, 4)) * 0.5).astype(np.float32)),
                      (F_DN_DT, FP32, 1, 32, rng.standard_normal((1, 32)).astype(np.float32)),
                      (F_DN_A, FP32, 1, 32, -np.exp(0.5 * rng.standard_normal((1, 32))).astype(np.float32)),
                      (F_DN_NORM, FP32, 1, 128, vec(128))]
            t += [(F_MOE_ROUTER, FP32, N_EXPERTS, HIDDEN,
                   (rng.standard_normal((N_EXPERTS, HIDDEN)) * 0.02).astype(np.float32))]
            if shared:
                t += [(F_SHARED_GATE, weight_quant, INTER, HIDDEN, mat(weight_quant, INTER, HIDDEN, ws)),
                      (F_SHARED_UP, weight_quant, INTER, HIDDEN, mat(weight_quant, INTER, HIDDEN, ws)),
                      (F_SHARED_DOWN, weight_quant, HIDDEN, INTER, mat(weight_quant, HIDDEN, INTER, ws * out_scale)),
                      (F_SHARED_ROUTER, FP32, 1, HIDDEN, (rng.standard_normal((1, HIDDEN)) * 0.02).astype(np.float32))]
            sets[a] = t
        for (f, q, r, c, arr) in sets[a]:
            m.add(f, l, q, r, c, arr)
        e = l % expert_period
        if e not in esets:
            esets[e] = tuple(make_matrix(expert_quant, N_EXPERTS * r, c, rng, es * sc)
                             for r, c, sc in ((INTER, HIDDEN, 1.0), (INTER, HIDDEN, 1.0), (HIDDEN, INTER, out_scale)))
        for f, (r, c), arr in zip((F_EXPERT_GATE, F_EXPERT_UP, F_EXPERT_DOWN),
                                  ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)), esets[e]):
            m.add(f, l, expert_quant, r, c, arr, r * row_bytes(expert_quant, c))
    m.add(F_TOK_EMBD, -1, weight_quant, embd_rows, HIDDEN, make_matrix(weight_quant, embd_rows, HIDDEN, rng, 1e-3))
    m.add(F_OUTPUT, -1, weight_quant, vocab, HIDDEN, mat(weight_quant, vocab, HIDDEN, ws))
    m.add(F_OUTPUT_NORM, -1, FP32, 1, HIDDEN, vec(HIDDEN))
    return m
