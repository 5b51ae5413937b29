"""The C-ABI library without a GPU: it loads, exports every declared symbol,
and rejects bad arguments before touching the device."""

import ctypes as C
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from tiktok_techjam_2026_track3_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "ttj_attn.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(ttj_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert set(declared_functions()) == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.ttj_version() >= 100
    assert lib.ttj_status_string(0) == b"ok"
    assert lib.ttj_status_string(-2) == b"unsupported shape or dtype"
    assert lib.ttj_status_string(-99) == b"unknown status"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
@pytest.mark.parametrize("cname,pyname", [("ttj_attn_layer_args", "AttnLayerArgs"),
                                          ("ttj_int8_attn_layer_args", "Int8AttnLayerArgs"),
                                          ("ttj_block_args", "BlockArgs")])
def test_struct_layout_matches_header(tmp_path, cname, pyname):
    """Every field offset of the ctypes mirror equals the C compiler's."""
    cls = getattr(_lib, pyname)
    fields = [f for f, _ in cls._fields_]
    src = tmp_path / "layout.c"
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
             f'printf("%zu\\n", sizeof({cname}));']
    lines += [f'printf("%zu\\n", offsetof({cname}, {f}));' for f in fields]
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    assert got[0] == C.sizeof(cls)
    assert got[1:] == [getattr(cls, f).offset for f in fields]


def test_argument_validation_without_device():
    lib = _lib.load()
    fake = 1 << 20  # never dereferenced: validation fails first
    # null pointers
    assert lib.ttj_linear_fwd(None, fake, fake, None, None, fake, 4, 32, 8, 0, None, None) == -1
    # bad dtype
    assert lib.ttj_linear_fwd(fake, fake, fake, None, None, fake, 4, 32, 8, 7, None, None) == -1
    # N not a multiple of 32
    assert lib.ttj_linear_fwd(fake, fake, fake, None, None, fake, 4, 48, 8, 0, None, None) == -2
    assert b"multiple of 32" in lib.ttj_last_error()
    # misaligned pointer
    assert lib.ttj_linear_fwd(fake + 2, fake, fake, None, None, fake, 4, 32, 8, 0, None, None) == -3
    # head_dim must be a multiple of 8 and at most 256 (12 and 264 are not)
    assert lib.ttj_flash_attn_fwd(fake, None, fake, 1, 16, 8, 12, 1, 0, None, None) == -2
    assert b"head_dim" in lib.ttj_last_error()
    assert lib.ttj_flash_attn_fwd(fake, None, fake, 1, 16, 2, 264, 1, 0, None, None) == -2
    assert b"head_dim" in lib.ttj_last_error()
    # d_model must be a multiple of 32 (head_dim 8 over 3 heads: d_model 24)
    assert lib.ttj_flash_attn_fwd(fake, None, fake, 1, 16, 3, 8, 1, 0, None, None) == -2
    assert b"multiple of 32" in lib.ttj_last_error()
    # factors beyond the limits are rejected before any product is formed (no wrap-around)
    assert lib.ttj_flash_attn_fwd(fake, None, fake, (1 << 57) + 1, 128, 4, 32, 1, 0, None, None) == -2
    assert lib.ttj_flash_attn_fwd(fake, None, fake, 1 << 30, 1 << 22, 32, 128, 1, 0, None, None) == -2
    assert b"too large" in lib.ttj_last_error()
    assert lib.ttj_attn_layer_workspace_size((1 << 57) + 1, 128, 128, 0) == 0
    # d_model not divisible by heads via the layer entry point
    a = _lib.AttnLayerArgs(x=fake, w_qkv=fake, b_qkv=fake, w_o=fake, b_o=fake, out=fake * 2,
                           workspace=fake, workspace_bytes=1 << 40, batch=1, seq_len=8,
                           d_model=129, num_heads=2, causal=1, dtype=0)
    assert lib.ttj_attn_layer_fwd(C.byref(a), None) == -1
    # workspace too small
    a.d_model = 128
    a.workspace_bytes = 16
    assert lib.ttj_attn_layer_fwd(C.byref(a), None) == -6
    # out aliasing x
    a.workspace_bytes = 1 << 40
    a.out = a.x
    assert lib.ttj_attn_layer_fwd(C.byref(a), None) == -1
    # int8 gemm needs K % 16
    assert lib.ttj_int8_gemm_s32(fake, fake, fake, 16, 32, 24, None, None) == -2
    # LayerNorm: d must be a multiple of 8 and at most 8192
    assert lib.ttj_layernorm_fwd(fake, fake, fake, None, fake, 4, 12, 1e-5, 0, None) == -2
    assert lib.ttj_layernorm_fwd(fake, fake, fake, None, fake, 4, 16384, 1e-5, 0, None) == -2
    assert lib.ttj_layernorm_fwd(None, fake, fake, None, fake, 4, 64, 1e-5, 0, None) == -1
    assert lib.ttj_linear_gelu_fwd(fake, fake, fake, fake, 4, 40, 8, 0, None, None) == -2
    # block: ffn_dim must be a multiple of 32, workspace must be large enough
    b = _lib.BlockArgs(**{f: fake for f in ("x", "ln1_w", "ln1_b", "w_qkv", "b_qkv", "w_o", "b_o",
                                            "ln2_w", "ln2_b", "w_in", "b_in", "w_out", "b_out")},
                       out=fake * 2, workspace=fake, workspace_bytes=1 << 40, batch=1, seq_len=8,
                       d_model=128, num_heads=2, ffn_dim=100, eps1=1e-5, eps2=1e-5, causal=1, dtype=0)
    assert lib.ttj_transformer_block_fwd(C.byref(b), None) == -2
    b.ffn_dim = 512
    b.workspace_bytes = 64
    assert lib.ttj_transformer_block_fwd(C.byref(b), None) == -6
    b.workspace_bytes = 1 << 40
    b.out = b.x
    assert lib.ttj_transformer_block_fwd(C.byref(b), None) == -1
    # fp32 residual stream (TTJ_F32): accepted by the block and LayerNorm only, d <= 4096
    b.out = fake * 2
    b.dtype = 2
    b.d_model, b.num_heads = 8192, 64
    assert lib.ttj_transformer_block_fwd(C.byref(b), None) == -2
    assert b"4096" in lib.ttj_last_error()
    assert lib.ttj_layernorm_fwd(fake, fake, fake, None, fake, 4, 8192, 1e-5, 2, None) == -2
    assert lib.ttj_layernorm_fwd(fake, fake, fake, None, fake, 4, 12, 1e-5, 2, None) == -2
    assert lib.ttj_linear_fwd(fake, fake, fake, None, None, fake, 4, 32, 8, 2, None, None) == -1
    assert lib.ttj_flash_attn_fwd(fake, None, fake, 1, 16, 2, 64, 1, 2, None, None) == -1


def test_workspace_sizes():
    lib = _lib.load()
    t, d = 8 * 2048, 1024
    assert lib.ttj_attn_layer_workspace_size(8, 2048, 1024, 0) == t * 3 * d * 2 + t * d * 2
    assert lib.ttj_attn_layer_workspace_size(0, 2048, 1024, 0) == 0
    assert lib.ttj_int8_attn_layer_workspace_size(1, 128, 256, 1) >= 128 * 256 * (1 + 6 + 2)
    # block: norm output, max(3D, F) wide buffer, context, x1
    assert lib.ttj_block_workspace_size(8, 2048, 1024, 4096, 0) == t * d * 2 * 3 + t * 4096 * 2
    assert lib.ttj_block_workspace_size(8, 2048, 1024, 1024, 0) == t * d * 2 * 3 + t * 3 * d * 2
    # fp32 residual stream: x1 is fp32
    assert lib.ttj_block_workspace_size(8, 2048, 1024, 4096, 2) == t * d * 2 * 2 + t * d * 4 + t * 4096 * 2


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="not found"):
        _lib.load(tmp_path / "nope.so")


def test_c_program_builds_against_the_abi(tmp_path):
    """tests/c/layer_check.c, which drives the whole layer from C, compiles
    with -Werror against include/ttj_attn.h and links against the library
    (it runs in tests/test_gpu_capi_c.py)."""
    from capi_c_build import build, toolchain_available
    if not toolchain_available():
        pytest.skip("gcc, the CUDA headers or the built library missing")
    assert build(tmp_path).exists()

