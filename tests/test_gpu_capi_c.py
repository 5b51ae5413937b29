"""The attention layer driven from a C program through the C ABI (no Python
or torch on the call path) against a double-precision restatement computed in
the same program; see tests/c/layer_check.c."""

import re
import subprocess

import pytest

from capi_c_build import build, toolchain_available

pytestmark = pytest.mark.gpu


def test_c_program_layer_matches_reference(tmp_path):
    if not toolchain_available():
        pytest.skip("gcc, the CUDA headers or the built library missing")
    exe = build(tmp_path)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    outside = [int(m) for m in re.findall(r"(\d+) of \d+ outside the predicate", res.stdout)]
    assert outside == [0] * 6, res.stdout
