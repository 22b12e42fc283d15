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
