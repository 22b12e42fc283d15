"""Helpers for the -m gpu tests: device buffers come from torch (plumbing
only); every computation goes through libqw6cuda's C ABI."""
import numpy as np


def torch():
    import torch as _t
    return _t


def dev(a: np.ndarray):
    t = torch()
    return t.from_numpy(np.ascontiguousarray(a)).cuda()


def empty_f32(*shape):
    t = torch()
    return t.empty(*shape, dtype=t.float32, device="cuda")


def sync(ctx):
    torch().cuda.synchronize()
    ctx.synchronize()


def host(t) -> np.ndarray:
    torch().cuda.synchronize()
    return t.cpu().numpy()


def pack(ctx, quant, raw: np.ndarray, rows: int, cols: int, count: int = 1):
    """Upload raw GGUF bytes of `count` matrices and pack them on the GPU.
    Returns (packed tensor, packed stride in bytes)."""
    t = torch()
    raw_d = dev(raw.reshape(-1).view(np.uint8))
    pb = ctx.packed_bytes(quant, rows, cols)
    stride = (pb + 255) // 256 * 256
    out = t.empty(stride * count, dtype=t.uint8, device="cuda")
    rb = raw.nbytes // count
    sync(ctx)
    ctx.pack(quant, raw_d.data_ptr(), out.data_ptr(), rows, cols, count, rb, stride)
    ctx.synchronize()
    return out, stride
