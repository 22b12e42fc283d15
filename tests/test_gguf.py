"""CPU: the library's GGUF reader (qw6cu_gguf_*) on synthetic GGUF v3 files.

The tensor table it reads must match what was written (names, dims, ggml
types, qw6 quant codes as qw6_gguf_to_quant maps them, qw6.c:1079-1094,
absolute offsets, data bytes) and what qw6's own reader prints for the same
file (`qw6 --inspect-gguf`, qw6.c:1243-1322, built from the reference
sources); malformed files are refused.  Nothing here touches a GPU."""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.gguf_util import GGML, KV_ARRAY, KV_F32, KV_STRING, KV_U32, write_gguf

ROOT = Path(__file__).resolve().parents[1]
QW6_CLI = ROOT / "oracle" / "_ref" / "qw6_cuda"
E, H, I = 8, 512, 256


def model_tensors(rng, layers=2):
    """Expert packs of `layers` MoE layers (Q4_K gate/up, Q6_K down, stored
    [cols, rows, experts] as qw6 expects, qw6.c:542-597) plus an fp32 router,
    an fp16 and a bf16 vector."""
    out = []
    for l in range(layers):
        g, u, d = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
        out += [(f"blk.{l}.ffn_gate_exps.weight", "Q4_K", [H, I, E], g),
                (f"blk.{l}.ffn_up_exps.weight", "Q4_K", [H, I, E], u),
                (f"blk.{l}.ffn_down_exps.weight", "Q6_K", [I, H, E], d),
                (f"blk.{l}.ffn_gate_inp.weight", "F32", [H, E], rng.standard_normal((E, H), dtype=np.float32))]
    out.append(("output_norm.weight", "F16", [H], rng.standard_normal(H).astype(np.float16)))
    out.append(("extra.bf16", "BF16", [H], S.bf16_round(rng.standard_normal(H).astype(np.float32))))
    return out


KV = [("general.architecture", KV_STRING, "qwen35moe"), ("qwen35moe.expert_count", KV_U32, E),
      ("qwen35moe.rope.freq_base", KV_F32, 1e7), ("tokenizer.ggml.tokens", KV_ARRAY, (KV_STRING, ["a", "bb", "c"]))]


@pytest.mark.parametrize("align", [None, 64])
def test_tensor_table_matches_what_was_written(tmp_path, rng, align):
    tensors = model_tensors(rng)
    path = tmp_path / "m.gguf"
    where = write_gguf(path, tensors, KV, alignment=align)
    g = L.Gguf(path)
    assert len(g) == len(tensors)
    quant = {"Q4_K": S.Q4_K, "Q6_K": S.Q6_K, "F32": S.FP32, "F16": S.FP16, "BF16": S.BF16}
    raw = path.read_bytes()
    for i, (name, tname, dims, data) in enumerate(tensors):
        info = g.info(i)
        assert info["name"] == name and info["dims"] == dims
        assert info["ggml_type"] == GGML[tname] and info["quant"] == quant[tname]
        _, abs_off, nbytes = where[name]
        assert info["file_offset"] == abs_off and info["bytes"] == nbytes
        assert raw[abs_off:abs_off + nbytes] == np.ascontiguousarray(data).tobytes()
        assert g.find(name) == i
    assert g.find("no.such.tensor") == -1
    # upload sizes: expert packs at a 256-aligned packed stride per expert
    i = g.find("blk.0.ffn_gate_exps.weight")
    assert g.upload_bytes(i) == E * ((L.Context.packed_bytes(S.Q4_K, I, H) + 255) // 256 * 256)
    g.close()


@pytest.mark.skipif(not QW6_CLI.exists(), reason="qw6's CLI not built (reference tree absent when building)")
def test_qw6_own_reader_agrees(tmp_path, rng):
    """qw6's --inspect-gguf (its own parser) reads the same alignment, data
    offset and tensor table (names, dims, offsets) from the file."""
    tensors = model_tensors(rng, layers=1)
    path = tmp_path / "m.gguf"
    write_gguf(path, tensors, KV, alignment=64)
    r = subprocess.run([str(QW6_CLI), "--inspect-gguf", str(path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    out = r.stdout
    g = L.Gguf(path)
    data_off = int(re.search(r"data_offset: (\d+)", out).group(1))
    assert int(re.search(r"alignment: (\d+)", out).group(1)) == 64
    rows = re.findall(r"\[\s*(\d+)\] (\S+)\s+\S+ \[([\d,]+)\] offset=(\d+)", out)
    assert len(rows) == len(tensors)
    for idx, name, dims, off in rows:
        info = g.info(int(idx))
        assert info["name"] == name
        assert info["dims"] == [int(d) for d in dims.split(",")]
        assert info["file_offset"] == data_off + int(off)


def test_malformed_files_are_refused(tmp_path, rng):
    tensors = model_tensors(rng, layers=1)
    good = tmp_path / "good.gguf"
    write_gguf(good, tensors, KV)
    raw = good.read_bytes()
    cases = {
        "magic": b"GGUX" + raw[4:],
        "version": raw[:4] + (2).to_bytes(4, "little") + raw[8:],
        "truncated_table": raw[:200],
        "truncated_data": raw[:-100],
    }
    for name, blob in cases.items():
        p = tmp_path / f"{name}.gguf"
        p.write_bytes(blob)
        with pytest.raises(L.Qw6CudaError):
            L.Gguf(p)
