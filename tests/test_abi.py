"""CPU: the C-ABI library loads, exports every symbol include/*.h declares,
the packed tile layout is a same-size bijection, and qw6.c links against the
drop-in header + library.  No compute call is made (no GPU here)."""
import ctypes
import os
import re
import shutil
import subprocess
import tempfile
from pathlib import Path

import pytest

from tests.conftest import REF_DIR

ROOT = Path(__file__).resolve().parents[1]
INCLUDE = ROOT / "include"
LIB = ROOT / "qw6_b200" / "libqw6cuda.so"
BUILD = ROOT / "_build"


def declared_functions():
    names = set()
    for h in INCLUDE.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(qw6\w+)\s*\(", text, re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_reference_surface():
    names = set(declared_functions())
    ref_h = REF_DIR / "qw6_vk.h"
    if ref_h.exists():
        ref_names = set(re.findall(r"\b(qw6_vk_\w+)\s*\(", ref_h.read_text()))
        assert ref_names <= names, sorted(ref_names - names)
    for n in ("qw6_vk_matmul_q4k_host", "qw6_vk_moe_route_host", "qw6cu_moe_decode", "qw6cu_matvec"):
        assert n in names


def test_library_exports_every_declared_symbol():
    if not LIB.exists():
        pytest.skip("libqw6cuda.so not built")
    lib = ctypes.CDLL(str(LIB))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True).stdout
    assert re.search(r"\bT qw6_vk_matmul_q4k_host\b", out)


def test_library_is_sm100a_only():
    if not LIB.exists():
        pytest.skip("libqw6cuda.so not built")
    out = subprocess.run(["cuobjdump", "--list-elf", str(LIB)], capture_output=True, text=True).stdout
    arches = set(re.findall(r"sm_(\d+a?)", out))
    assert arches == {"100a"}, arches


def test_packed_layout_is_a_bijection():
    """Host-side check of Fmt<F>::dst for every format (compiled by nvcc,
    run on the CPU)."""
    src = ROOT / "tests" / "csrc" / "check_pack_layout.cu"
    BUILD.mkdir(exist_ok=True)
    exe = BUILD / "check_pack_layout"
    subprocess.run(["nvcc", "-std=c++17", "-O1", "-I", str(ROOT / "qw6_b200" / "csrc"), str(src), "-o", str(exe)],
                   check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all layouts ok" in r.stdout


@pytest.mark.skipif(not (REF_DIR / "qw6.c").exists(), reason="reference tree absent")
def test_qw6_links_against_dropin_library():
    """qw6.c built with -DQW6_VULKAN links against include/qw6_vk.h and
    libqw6cuda.so unchanged.  The reference files are linked into a scratch
    dir (symlinks, not copies) that omits qw6's own qw6_vk.h."""
    if not LIB.exists():
        pytest.skip("libqw6cuda.so not built")
    with tempfile.TemporaryDirectory() as td:
        for f in ("qw6.c", "qw6.h", "qw6_tok.c", "qw6_tok.h", "qw6_iq_tables.h"):
            os.symlink(REF_DIR / f, Path(td) / f)
        exe = Path(td) / "qw6_cuda"
        cmd = [shutil.which("gcc") or "gcc", "-std=c11", "-O1", "-DQW6_VULKAN", "-I", str(INCLUDE),
               str(Path(td) / "qw6.c"), str(Path(td) / "qw6_tok.c"), "-o", str(exe), "-L", str(LIB.parent),
               "-lqw6cuda", "-lm", f"-Wl,-rpath,{LIB.parent}"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-3000:]
        assert exe.exists()


@pytest.mark.skipif(not (REF_DIR / "qw6.h").exists(), reason="reference tree absent")
def test_model_layout_matches_qw6():
    """qw6_model_abi.h (the pipeline's view of qw6_model_t) has the layout of
    qw6.h's structs as qw6 is built with QW6_VULKAN: a C file that includes
    both compiles only if every offset the pipeline reads matches."""
    fields = ("norm", "post_norm", "attn_q", "attn_k", "attn_v", "attn_o", "attn_q_norm", "attn_k_norm",
              "attn_gate", "conv1d", "dn_out", "dn_norm", "dn_alpha", "dn_beta", "dn_dt", "dn_a", "moe_router",
              "shared_router", "expert_gate[0]", "expert_up[17]", "expert_down[255]", "shared_gate", "shared_up",
              "shared_down")
    checks = ["_Static_assert(sizeof(qw6_tensor_t) == sizeof(qw6abi_tensor), \"tensor size\");"]
    for f in ("name", "rows", "cols", "quant", "data", "vk_offset"):
        checks.append(f"_Static_assert(offsetof(qw6_tensor_t, {f}) == offsetof(qw6abi_tensor, {f}), \"{f}\");")
    for top in ("tok_embeddings", "output", "output_norm", "max_context"):
        checks.append(f"_Static_assert(offsetof(qw6_model_t, {top}) == offsetof(qw6abi_model, {top}), \"{top}\");")
    for layer in (0, 3, 39):
        for f in fields:
            p = f"layers[{layer}].{f}"
            checks.append(f"_Static_assert(offsetof(qw6_model_t, {p}) == offsetof(qw6abi_model, {p}), \"{p}\");")
    src = ("#define QW6_VULKAN 1\n#include <stddef.h>\n#include \"qw6.h\"\n#include \"qw6_model_abi.h\"\n"
           + "\n".join(checks) + "\nint main(void) { return 0; }\n")
    with tempfile.TemporaryDirectory() as td:
        c = Path(td) / "layout.c"
        c.write_text(src)
        r = subprocess.run([shutil.which("gcc") or "gcc", "-std=c11", "-fsyntax-only", "-I", str(REF_DIR), "-I",
                            str(ROOT / "qw6_b200" / "csrc"), str(c)], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-3000:]
