"""The int8 activation quantiser's element arithmetic, checked on the CPU.

The kernel (csrc/quant_rows.cu) replaces the recipe's per-element IEEE
division x / s (Project/kernels/k008_int8_gemm.py:148-151) by a correctly
rounded reciprocal of s with one residual correction, and rounds half-to-even
by adding 1.5 * 2^23.  tests/c/quant_div_check.c evaluates both forms in
fp32 with fused multiply-adds (as the GPU does) and compares them.  Run with
stride 1 it covers every scale a row of 16-bit values can produce; here a
strided subset keeps the CPU suite fast (a full run takes ~45 s).
"""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "c" / "quant_div_check.c"


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    exe = tmp_path_factory.mktemp("qdc") / "quant_div_check"
    # no contraction: only the fused steps written as fmaf() may fuse
    subprocess.run(["gcc", "-std=c11", "-O2", "-ffp-contract=off", "-Wall", "-Wextra", "-Werror",
                    str(SRC), "-o", str(exe), "-lm"], check=True)
    return exe


@pytest.mark.parametrize("dtype,first", [("f16", 0), ("f16", 7), ("bf16", 0), ("bf16", 11)])
def test_quantiser_quotient_and_rounding_match_ieee(checker, dtype, first):
    res = subprocess.run([str(checker), dtype, "41", str(first)], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "0 int8 mismatches" in res.stdout
