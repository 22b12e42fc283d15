#!/usr/bin/env python3
"""Generate tests/golden/*.npz from qw6's OWN CPU code.

Runs in the build container, where the reference tree exists and
oracle/_ref/libqw6ref.so has been compiled from its sources (oracle/Makefile).
The fixtures carry qw6's outputs so that the parity tests can pin the oracle
and the CUDA library on machines without the reference tree:

  matvec_<fmt>.npz  raw GGUF bytes (seeded random rows + rows whose fp16
                    scales are 0, -0, subnormal, max, +-inf, NaN), x,
                    qw6_tensor_dequantize_row output, qw6_tensor_matvec output
  route.npz         qw6_cpu_moe_route on random / tied / -inf / NaN logits
  argmax.npz        qw6_cpu_argmax cases
  moe_small.npz     qw6_apply_layer_moe composition (qw6.c:2246-2264) for a
                    4-expert layer whose weights are regenerated from the seed
                    (their sha256 is stored to detect generator drift)
  moe_block.npz     the full MoE FFN block (qw6.c:2474-2484 around
                    qw6.c:2226-2290: RMSNorm, fp32 router, routed experts,
                    shared expert with its sigmoid gate, residual add), weights
                    regenerated from the seed by block_inputs() and checked by
                    sha256
  sample.npz        qw6_sample on full-vocabulary logit rows regenerated from a
                    seed by sample_logits(), for several (temp, top_p, top_k)
                    and libc rand() seeds, with the uniform draw each made

Usage: python tests/golden/gen_golden.py
"""
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle.oracle import Reference  # noqa: E402
from qw6_b200 import synth as S  # noqa: E402

SPECIAL_D = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x7E00, 0x3C00, 0xBC00]


def matvec_case(ref, q, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    rows, cols = 16, 512
    w = S.make_matrix(q, rows, cols, rng)
    sw = S.make_matrix(q, len(SPECIAL_D), cols, rng).reshape(len(SPECIAL_D), cols // 256, -1)
    o = 208 if q == S.Q6_K else 0
    for r, d in enumerate(SPECIAL_D):
        sw[r, :, o], sw[r, :, o + 1] = d & 0xFF, d >> 8
    sw = sw.reshape(len(SPECIAL_D), -1)
    x = rng.standard_normal(cols, dtype=np.float32)
    return dict(
        quant=np.int32(q), rows=np.int32(rows), cols=np.int32(cols), w=w, x=x,
        deq=ref.dequantize(q, w, rows, cols), y=ref.matvec(q, w, x, rows, cols),
        w_special=sw, deq_special=ref.dequantize(q, sw, len(SPECIAL_D), cols),
    )


def route_case(ref):
    rng = np.random.Generator(np.random.PCG64(11))
    L = []
    for t in range(48):
        lg = rng.standard_normal(256).astype(np.float32)
        if t % 3 == 0:
            lg[rng.integers(0, 256, 6)] = lg.max()
        if t % 4 == 0:
            lg = (np.round(lg * 2) / 2).astype(np.float32)
        L.append(lg)
    lg = np.full(256, -np.inf, np.float32)
    lg[[3, 9, 200]] = [1.0, 2.0, 3.0]
    L.append(lg)
    lg = np.linspace(-1, 1, 256).astype(np.float32)
    lg[0] = np.nan
    L.append(lg)
    lg = np.linspace(-1, 1, 256).astype(np.float32)
    lg[17] = np.nan
    L.append(lg)
    L.append(np.zeros(256, np.float32))
    logits = np.stack(L)
    idx = np.stack([ref.moe_route(lg, 8)[0] for lg in logits])
    w = np.stack([ref.moe_route(lg, 8)[1] for lg in logits])
    return dict(logits=logits, idx=idx, w=w)


def argmax_case(ref):
    rng = np.random.Generator(np.random.PCG64(12))
    xs = [rng.standard_normal(4097).astype(np.float32) for _ in range(4)]
    x = np.round(rng.standard_normal(10000) * 2).astype(np.float32)
    xs.append(x)
    x = rng.standard_normal(3000).astype(np.float32)
    x[0] = np.nan
    xs.append(x)
    x = rng.standard_normal(3000).astype(np.float32)
    x[5] = np.nan
    xs.append(x)
    xs.append(np.full(257, -np.inf, np.float32))
    n = max(len(v) for v in xs)
    pad = np.full((len(xs), n), np.nan, np.float32)
    lens = np.array([len(v) for v in xs], np.int32)
    for i, v in enumerate(xs):
        pad[i, :len(v)] = v
    return dict(x=pad, n=lens, idx=np.array([ref.argmax(v) for v in xs], np.int32))


def moe_case(ref):
    seed, E, H, I, K, T = 21, 4, 512, 512, 2, 3
    rng = np.random.Generator(np.random.PCG64(seed))
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    out, idx, w = ref.moe_layer(S.Q4_K, gate, up, S.Q6_K, down, logits, x, top_k=K)
    sha = hashlib.sha256(gate.tobytes() + up.tobytes() + down.tobytes()).hexdigest()
    return dict(seed=np.int32(seed), dims=np.array([E, H, I, K, T], np.int32), sha=np.array(sha),
                logits=logits, x=x, out=out, idx=idx, w=w)


def block_inputs(seed):
    """Inputs of the moe_block fixture, all drawn from one seeded generator:
    x [T x H], norm_w [H], the fp32 router [E x H], the routed experts
    (Q4_K gate/up [I x H], Q6_K down [H x I]) and the shared expert (Q4_K
    gate/up [SI x H], Q6_K down [H x SI], fp32 router [1 x H])."""
    E, H, I, SI, K, T = 4, 512, 256, 256, 2, 3
    rng = np.random.Generator(np.random.PCG64(seed))
    gate, up, down = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
    router = (rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    sg, su = S.make_matrix(S.Q4_K, SI, H, rng), S.make_matrix(S.Q4_K, SI, H, rng)
    sd = S.make_matrix(S.Q6_K, H, SI, rng)
    sr = (rng.standard_normal((1, H), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    norm_w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    experts = (S.Q4_K, gate, up, S.Q6_K, down)
    shared = ((S.Q4_K, sg), (S.Q4_K, su), (S.Q6_K, sd), (S.FP32, sr))
    sha = hashlib.sha256(b"".join(a.tobytes() for a in (gate, up, down, router, sg, su, sd, sr, norm_w, x)))
    return dict(dims=(E, H, I, SI, K, T), x=x, norm_w=norm_w, router=(S.FP32, router), experts=experts,
                shared=shared, sha=sha.hexdigest())


def block_case(ref):
    seed = 22
    b = block_inputs(seed)
    K = b["dims"][4]
    out = ref.moe_block(b["x"], b["norm_w"], b["router"], b["experts"], b["shared"], top_k=K)
    routed = ref.moe_block(b["x"], b["norm_w"], b["router"], b["experts"], None, top_k=K)
    return dict(seed=np.int32(seed), sha=np.array(b["sha"]), out=out, out_routed=routed)


SAMPLE_PARAMS = [(0.0, 1.0, 0), (1.0, 1.0, 0), (0.7, 0.9, 40), (1.3, 0.5, 0), (1.0, 1.0, 1), (0.8, 1.0, 50),
                 (1.0, 0.95, 0)]


def sample_logits(seed, vocab):
    """One logit row of the sample fixture: N(0, 3) with 8 tied maxima."""
    rng = np.random.Generator(np.random.PCG64(seed))
    logits = (rng.standard_normal(vocab) * 3.0).astype(np.float32)
    logits[rng.integers(0, vocab, 8)] = logits.max()
    return logits


def sample_case(ref):
    rows = []
    for i, (temp, top_p, top_k) in enumerate(SAMPLE_PARAMS):
        logits = sample_logits(300 + i, ref.vocab)
        for rseed in (1, 7, 12345):
            rows.append((300 + i, temp, top_p, top_k, rseed, ref.rand_unit(rseed),
                         ref.sample(logits, temp, top_p, top_k, rseed)))
    a = np.array(rows, dtype=np.float64)
    sha = hashlib.sha256(sample_logits(300, ref.vocab).tobytes()).hexdigest()
    return dict(vocab=np.int32(ref.vocab), cases=a, sha=np.array(sha))


def main():
    ref = Reference()
    for i, q in enumerate(S.BLOCK_QUANTS):
        np.savez_compressed(HERE / f"matvec_{S.QUANT_NAMES[q]}.npz", **matvec_case(ref, q, 100 + i))
    np.savez_compressed(HERE / "route.npz", **route_case(ref))
    np.savez_compressed(HERE / "argmax.npz", **argmax_case(ref))
    np.savez_compressed(HERE / "moe_small.npz", **moe_case(ref))
    np.savez_compressed(HERE / "moe_block.npz", **block_case(ref))
    np.savez_compressed(HERE / "sample.npz", **sample_case(ref))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
