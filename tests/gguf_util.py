"""Writer of small GGUF (v3) files for the tests: the public GGUF layout --
little-endian header (magic "GGUF", version 3, tensor count, metadata
count), metadata (key string, type, value), tensor table (name, dims,
ggml type, offset into the data section), then the tensor data from an
offset aligned to general.alignment (default 32), each tensor aligned too."""
from __future__ import annotations

import struct

import numpy as np

# ggml type ids (qw6.h:346-379) of the formats the library handles
GGML = {"F32": 0, "F16": 1, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16, "IQ3_S": 21, "IQ2_S": 22,
        "BF16": 30, "Q8_0": 8}
# metadata value types
KV_U32, KV_I32, KV_F32, KV_STRING, KV_ARRAY, KV_U64 = 4, 5, 6, 8, 9, 10


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, value) -> bytes:
    out = _str(key) + struct.pack("<I", vtype)
    if vtype == KV_STRING:
        return out + _str(value)
    if vtype == KV_ARRAY:
        etype, items = value
        out += struct.pack("<IQ", etype, len(items))
        if etype == KV_STRING:
            return out + b"".join(_str(v) for v in items)
        fmt = {KV_U32: "<I", KV_I32: "<i", KV_F32: "<f", KV_U64: "<Q"}[etype]
        return out + b"".join(struct.pack(fmt, v) for v in items)
    fmt = {KV_U32: "<I", KV_I32: "<i", KV_F32: "<f", KV_U64: "<Q"}[vtype]
    return out + struct.pack(fmt, value)


def write_gguf(path, tensors, kv=(), alignment: int | None = None) -> dict:
    """tensors: (name, ggml type name, dims [cols, rows, ...], uint8 data).
    Returns {name: (offset from the data section, data offset, bytes)}."""
    kvs = list(kv)
    if alignment is not None:
        kvs.append(("general.alignment", KV_U32, alignment))
    align = alignment or 32
    infos, blobs, where, off = [], [], {}, 0
    for name, tname, dims, data in tensors:
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        off = (off + align - 1) // align * align
        infos.append(_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
                     + struct.pack("<IQ", GGML[tname], off))
        blobs.append((off, data))
        where[name] = [off, None, data.size]
        off += data.size
    head = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kvs)) + b"".join(_kv(*k) for k in kvs) + b"".join(infos)
    data_off = (len(head) + align - 1) // align * align
    with open(path, "wb") as f:
        f.write(head + b"\0" * (data_off - len(head)))
        pos = 0
        for o, d in blobs:
            f.write(b"\0" * (o - pos))
            f.write(d.tobytes())
            pos = o + d.size
    for name in where:
        where[name][1] = data_off + where[name][0]
    return {k: tuple(v) for k, v in where.items()}
