"""Small, self-contained workloads for profiling one kernel under ncu.

    python -m qw6_b200.prof matvec <quant> <rows> <cols> [reps] [ntok]
    python -m qw6_b200.prof moe_decode <config> [layers] [steps]
    python -m qw6_b200.prof lm_head <ntok> [reps]
    python -m qw6_b200.prof decoder <tokens> [layers]

matvec: `reps` (default 5) launches of the packed quantized matvec
(qw6cu_matvec) over `ntok` tokens (default 1) on `rows` x `cols` random packed
bytes of the given format (q4k, q5k, q6k, iq2xxs, iq2s, iq3s); pick rows so
that the matrix is larger than L2 (126 MB) and a few hundred MB at most, and
capture with `-k regex:k_matvec -s 2 -c 1`.

moe_decode: `steps` (default 12) routed-MoE decode layers (qw6cu_moe_decode)
of configuration 1 (1 token, Q4_K gate/up, Q6_K down) or 2 (64 tokens,
IQ2_XXS) over `layers` (default 4) resident copies of the 256-expert layer,
step s using copy s % layers, so that consecutive launches read different
weights; 1 copy of config 1 is 0.5 GB, of config 2 0.2 GB.

lm_head: `reps` launches of config 4's fused Q6_K LM head + argmax
(248320 x 2048) over `ntok` tokens.

decoder: `tokens` greedy steps of the decode-step executor
(qw6cu_decoder_generate) on a full-size synthetic qw6 model (40 layers with
distinct weights, 248320-token vocabulary; 10.6 GB on the device, ~16 s to
generate on the host); each step is one CUDA graph of ~425 launches.
`layers` (default 40) fewer layers for captures that replay a kernel
(4 layers: ~1.2 GB on the device).

The values are random, so the outputs are meaningless; only the kernels'
work is real.
"""
from __future__ import annotations

import sys


def matvec(quant: str, rows: int, cols: int, reps: int = 5, ntok: int = 1) -> None:
    import torch

    from . import lib as L
    from . import synth as S
    q = {v: k for k, v in S.QUANT_NAMES.items()}[quant]
    ctx = L.Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream or 1)
    w = torch.randint(0, 256, (ctx.packed_bytes(q, rows, cols),), dtype=torch.uint8, device="cuda")
    x = torch.randn(ntok, cols, device="cuda")
    y = torch.empty(ntok, rows, device="cuda")
    torch.cuda.synchronize()
    for _ in range(reps):
        ctx.matvec(q, w.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, ntok)
    torch.cuda.synchronize()
    ctx.check_device_errors()
    print(f"matvec {quant} {rows}x{cols} ntok {ntok}: {reps} launches")


def moe_decode(config: int, layers: int = 4, steps: int = 12) -> None:
    import numpy as np
    import torch

    from . import lib as L
    from . import synth as S
    H, I, E, K = S.HIDDEN, S.INTER, S.N_EXPERTS, S.TOP_K
    if config == 1:
        ntok, gq, dq = 1, S.Q4_K, S.Q6_K
    elif config == 2:
        ntok, gq, dq = 64, S.IQ2_XXS, S.IQ2_XXS
    else:
        raise SystemExit("moe_decode: config is 1 or 2")
    rng = np.random.Generator(np.random.PCG64(config))
    ctx = L.Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream or 1)
    copies = []
    for q, r, c in ((gq, I, H), (gq, I, H), (dq, H, I)):
        pb = ctx.packed_bytes(q, r, c)
        # random packed bytes with well-formed fp16 scales are not needed for timing
        t = torch.randint(0, 256, (layers, pb * E), dtype=torch.uint8, device="cuda")
        copies.append((q, pb, t))
    logits = torch.from_numpy(rng.standard_normal((ntok, E), dtype=np.float32)).cuda()
    x = torch.from_numpy(rng.standard_normal((ntok, H), dtype=np.float32)).cuda()
    out = torch.empty((ntok, H), device="cuda")
    torch.cuda.synchronize()
    for s in range(steps):
        g, u, d = (L.ExpertPack(q, t[s % layers].data_ptr(), pb) for q, pb, t in copies)
        ctx.moe_decode(g, u, d, logits.data_ptr(), x.data_ptr(), out.data_ptr(), ntok, H, I, E, K)
    torch.cuda.synchronize()
    ctx.check_device_errors()
    print(f"moe_decode config {config}: {steps} layer steps over {layers} copies")


def lm_head(ntok: int, reps: int = 5) -> None:
    import torch

    from . import lib as L
    from . import synth as S
    rows, cols = S.VOCAB, S.HIDDEN
    ctx = L.Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream or 1)
    w = torch.randint(0, 256, (ctx.packed_bytes(S.Q6_K, rows, cols),), dtype=torch.uint8, device="cuda")
    x = torch.randn(ntok, cols, device="cuda")
    keys = torch.zeros(ntok, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    for _ in range(reps):
        ctx.lm_head_argmax(S.Q6_K, w.data_ptr(), x.data_ptr(), ntok, rows, cols, 0, keys.data_ptr())
    torch.cuda.synchronize()
    ctx.check_device_errors()
    print(f"lm_head ntok {ntok}: {reps} launches")


def decoder(tokens: int = 3, layers: int = 40) -> None:
    from qw6_b200 import lib as L
    from qw6_b200 import synth as S
    m = S.fwd_model(seed=31, n_layers=layers, vocab=S.VOCAB, embd_rows=S.VOCAB, attn_period=40, expert_period=40)
    ctx = L.Context(0)
    dec = L.Decoder(ctx, m, max_ctx=4096)
    del m
    print("decoder: picked", list(dec.generate(1, 0, tokens)))
    dec.close()
    ctx.close()


def main(argv: list[str]) -> int:
    if len(argv) >= 4 and argv[0] == "matvec":
        matvec(argv[1], int(argv[2]), int(argv[3]), *(int(a) for a in argv[4:6]))
        return 0
    if len(argv) >= 2 and argv[0] == "moe_decode":
        moe_decode(*(int(a) for a in argv[1:4]))
        return 0
    if len(argv) >= 2 and argv[0] == "lm_head":
        lm_head(*(int(a) for a in argv[1:3]))
        return 0
    if len(argv) >= 1 and argv[0] == "decoder":
        decoder(*(int(a) for a in argv[1:3]))
        return 0
    print(__doc__)
    return 2


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
