"""Small, self-contained workloads for profiling one kernel under ncu.

    python -m qw6_b200.prof matvec <quant> <rows> <cols> [reps]

runs `reps` (default 5) launches of the packed quantized matvec
(qw6cu_matvec, batch 1) on `rows` x `cols` random packed bytes of the given
format (q4k, q5k, q6k, iq2xxs, iq2s, iq3s) and one fp32 activation vector;
pick rows so that the matrix is larger than L2 (126 MB) and a few hundred MB
at most, and capture with `-k regex:k_matvec -s 2 -c 1`.  The values are
random, so the output is meaningless; only the kernel's work is real.
"""
from __future__ import annotations

import sys


def matvec(quant: str, rows: int, cols: int, reps: int = 5) -> None:
    import torch

    from . import lib as L
    from . import synth as S
    q = {v: k for k, v in S.QUANT_NAMES.items()}[quant]
    ctx = L.Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream or 1)
    w = torch.randint(0, 256, (ctx.packed_bytes(q, rows, cols),), dtype=torch.uint8, device="cuda")
    x = torch.randn(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    torch.cuda.synchronize()
    for _ in range(reps):
        ctx.matvec(q, w.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    ctx.check_device_errors()
    print(f"matvec {quant} {rows}x{cols}: {reps} launches")


def main(argv: list[str]) -> int:
    if len(argv) >= 4 and argv[0] == "matvec":
        matvec(argv[1], int(argv[2]), int(argv[3]), int(argv[4]) if len(argv) > 4 else 5)
        return 0
    print(__doc__)
    return 2


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
