"""ctypes binding of libttj_attn_sm100.so (the C ABI of include/ttj_attn.h).

The library is built in-tree by ``build_lib.py``.  There is no fallback: if
the library is missing or fails to load, every op raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path
from typing import Optional

LIB_PATH = Path(__file__).resolve().parent / "libttj_attn_sm100.so"

TTJ_F16 = 0
TTJ_BF16 = 1
TTJ_F32 = 2

STATUS_NAMES = {
    0: "TTJ_OK", -1: "TTJ_ERR_INVALID_ARG", -2: "TTJ_ERR_UNSUPPORTED",
    -3: "TTJ_ERR_ALIGNMENT", -4: "TTJ_ERR_CUDA", -5: "TTJ_ERR_DEVICE_TIMEOUT",
    -6: "TTJ_ERR_WORKSPACE",
}

# Every symbol include/ttj_attn.h declares (tests check the library exports them).
EXPORTED_SYMBOLS = (
    "ttj_version", "ttj_status_string", "ttj_last_error", "ttj_read_status",
    "ttj_selftest_wait_timeout",
    "ttj_linear_fwd", "ttj_linear_kchunked_fwd", "ttj_qkv_proj_fwd", "ttj_flash_attn_fwd", "ttj_out_proj_residual_fwd",
    "ttj_attn_layer_workspace_size", "ttj_attn_layer_fwd", "ttj_attn_layer_fwd_noalloc",
    "ttj_int8_quant_rows", "ttj_int8_gemm_s32", "ttj_int8_linear_fwd",
    "ttj_int8_attn_layer_workspace_size", "ttj_int8_attn_layer_fwd",
    "ttj_layernorm_fwd", "ttj_linear_gelu_fwd", "ttj_block_workspace_size", "ttj_transformer_block_fwd",
)

vp = C.c_void_p
i64 = C.c_int64
ci = C.c_int


class AttnLayerArgs(C.Structure):
    """Mirror of ``ttj_attn_layer_args``."""
    _fields_ = [
        ("x", vp), ("w_qkv", vp), ("b_qkv", vp), ("w_o", vp), ("b_o", vp),
        ("valid_token_mask", vp), ("residual", vp), ("out", vp),
        ("workspace", vp), ("workspace_bytes", C.c_size_t), ("status", vp),
        ("batch", i64), ("seq_len", i64), ("d_model", i64), ("num_heads", i64),
        ("causal", ci), ("dtype", ci),
    ]


class Int8AttnLayerArgs(C.Structure):
    """Mirror of ``ttj_int8_attn_layer_args``."""
    _fields_ = [
        ("x", vp), ("w_qkv", vp), ("s_qkv", vp), ("b_qkv", vp),
        ("w_o", vp), ("s_o", vp), ("b_o", vp),
        ("valid_token_mask", vp), ("residual", vp), ("out", vp),
        ("workspace", vp), ("workspace_bytes", C.c_size_t), ("status", vp),
        ("batch", i64), ("seq_len", i64), ("d_model", i64), ("num_heads", i64),
        ("causal", ci), ("dtype", ci),
    ]


class BlockArgs(C.Structure):
    """Mirror of ``ttj_block_args``."""
    _fields_ = [
        ("x", vp), ("ln1_w", vp), ("ln1_b", vp), ("w_qkv", vp), ("b_qkv", vp),
        ("w_o", vp), ("b_o", vp), ("ln2_w", vp), ("ln2_b", vp),
        ("w_in", vp), ("b_in", vp), ("w_out", vp), ("b_out", vp),
        ("valid_token_mask", vp), ("out", vp),
        ("workspace", vp), ("workspace_bytes", C.c_size_t), ("status", vp),
        ("batch", i64), ("seq_len", i64), ("d_model", i64), ("num_heads", i64), ("ffn_dim", i64),
        ("eps1", C.c_float), ("eps2", C.c_float),
        ("causal", ci), ("dtype", ci),
    ]


_SIGNATURES = {
    "ttj_version": (ci, []),
    "ttj_status_string": (C.c_char_p, [ci]),
    "ttj_last_error": (C.c_char_p, []),
    "ttj_read_status": (ci, [vp, C.POINTER(ci), vp]),
    "ttj_selftest_wait_timeout": (ci, [vp, i64, vp]),
    "ttj_linear_fwd": (ci, [vp, vp, vp, vp, vp, vp, i64, i64, i64, ci, vp, vp]),
    "ttj_linear_kchunked_fwd": (ci, [vp, i64, vp, vp, vp, vp, vp, i64, i64, i64, ci, vp, vp]),
    "ttj_qkv_proj_fwd": (ci, [vp, vp, vp, vp, i64, i64, ci, vp, vp]),
    "ttj_flash_attn_fwd": (ci, [vp, vp, vp, i64, i64, i64, i64, ci, ci, vp, vp]),
    "ttj_out_proj_residual_fwd": (ci, [vp, vp, vp, vp, vp, vp, i64, i64, ci, vp, vp]),
    "ttj_attn_layer_workspace_size": (C.c_size_t, [i64, i64, i64, ci]),
    "ttj_attn_layer_fwd": (ci, [C.POINTER(AttnLayerArgs), vp]),
    "ttj_attn_layer_fwd_noalloc": (ci, [C.POINTER(AttnLayerArgs), vp]),
    "ttj_int8_quant_rows": (ci, [vp, vp, vp, i64, i64, ci, vp]),
    "ttj_int8_gemm_s32": (ci, [vp, vp, vp, i64, i64, i64, vp, vp]),
    "ttj_int8_linear_fwd": (ci, [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, ci, vp, vp]),
    "ttj_int8_attn_layer_workspace_size": (C.c_size_t, [i64, i64, i64, ci]),
    "ttj_int8_attn_layer_fwd": (ci, [C.POINTER(Int8AttnLayerArgs), vp]),
    "ttj_layernorm_fwd": (ci, [vp, vp, vp, vp, vp, i64, i64, C.c_float, ci, vp]),
    "ttj_linear_gelu_fwd": (ci, [vp, vp, vp, vp, i64, i64, i64, ci, vp, vp]),
    "ttj_block_workspace_size": (C.c_size_t, [i64, i64, i64, i64, ci]),
    "ttj_transformer_block_fwd": (ci, [C.POINTER(BlockArgs), vp]),
}

_lock = threading.Lock()
_lib: Optional[C.CDLL] = None


def load(path: Optional[Path] = None) -> C.CDLL:
    """Load (once) and return the library with argtypes set.  Raises
    RuntimeError with the build command if it is missing."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"CUDA library {p.name} not found next to the package; build it with "
                "`python -m tiktok_techjam_2026_track3_b200.build_lib` (nvcc, sm_100a)")
        lib = C.CDLL(str(p))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    """Turn a ttj_status into a RuntimeError carrying ttj_last_error()."""
    if rc != 0:
        detail = load().ttj_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed: {STATUS_NAMES.get(rc, rc)}: {detail}")
