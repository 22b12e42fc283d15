"""CPU: the IQ codebooks and sign tables the kernels use equal qw6's."""
import importlib.util
import re
from pathlib import Path

import pytest

from tests.conftest import REF_DIR

ROOT = Path(__file__).resolve().parents[1]
GEN = ROOT / "qw6_b200" / "csrc" / "gen_iq_tables.py"
GRIDS_H = ROOT / "qw6_b200" / "csrc" / "qw6_iq_grids.h"


def _gen():
    spec = importlib.util.spec_from_file_location("gen_iq_tables", GEN)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.skipif(not (REF_DIR / "qw6_iq_tables.h").exists(), reason="reference tree absent")
def test_generated_grids_match_reference_header():
    assert _gen().generate(REF_DIR / "qw6_iq_tables.h") == GRIDS_H.read_text()


@pytest.mark.skipif(not (REF_DIR / "qw6_iq_tables.h").exists(), reason="reference tree absent")
def test_ksigns_formula_matches_reference_table():
    text = (REF_DIR / "qw6_iq_tables.h").read_text()
    body = re.search(r"ksigns_iq2xs\[128\]\s*=\s*\{(.*?)\};", text, re.S).group(1)
    table = [int(v) for v in re.findall(r"\d+", body)]
    formula = [i | ((bin(i).count("1") & 1) << 7) for i in range(128)]
    assert table == formula


def test_grid_value_sets():
    """Every grid byte is one of the IQ magnitudes (int8-exact for the MMAs)."""
    text = GRIDS_H.read_text()
    for name, allowed in (("IQ2XXS", {8, 25, 43}), ("IQ2S", {8, 25, 43}), ("IQ3S", {1, 3, 5, 7, 9, 11, 13, 15})):
        body = re.search(r"QW6_%s_GRID_BYTES_INIT \{(.*?)\}" % name, text, re.S).group(1)
        vals = {int(v, 16) for v in re.findall(r"0x[0-9a-f]{2}", body)}
        assert vals <= allowed, name
