"""GPU: the drop-in proven end to end.  qw6's own command-line program,
compiled from the reference sources with -DQW6_VULKAN against
include/qw6_vk.h and linked with libqw6cuda.so instead of qw6's Vulkan
backend (oracle/Makefile, target _ref/qw6_cuda), runs its Vulkan self-test
(`qw6 --vulkan-self-test`, qw6.c:3529-3540 -> qw6_vk_selftest) on the B200:
qw6's closed-form known-answer checks of the quantized matvecs, routing,
gather and argmax (qw6_vk.c:1609-1954) through this library."""
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
EXE = ROOT / "oracle" / "_ref" / "qw6_cuda"


def test_qw6_cli_vulkan_self_test_runs_on_this_library():
    if not EXE.exists():
        pytest.skip("oracle/_ref/qw6_cuda not built (the reference tree was absent when building)")
    r = subprocess.run([str(EXE), "--vulkan-self-test"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert "qw6cuda selftest: passed" in r.stderr, r.stderr[-3000:]
