"""Torch-facing wrappers over the C ABI: tensors in, tensors out, no fallback.

Every op checks device / dtype / contiguity, launches on the caller's current
CUDA stream through ``libttj_attn_sm100.so`` and raises ``RuntimeError`` on
any error code.  Nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, Optional, Tuple

import torch

from . import _lib

_DTYPES = {torch.float16: _lib.TTJ_F16, torch.bfloat16: _lib.TTJ_BF16}
_status_words: Dict[int, torch.Tensor] = {}


def _dtype_code(t: torch.Tensor) -> int:
    code = _DTYPES.get(t.dtype)
    if code is None:
        raise RuntimeError(f"unsupported dtype {t.dtype}: the sm_100a kernels take float16 or bfloat16")
    return code


def _cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (got {t.device}); there is no CPU path")
    if not t.is_contiguous():
        t = t.contiguous()
    return t


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word the kernels write on a bounded-wait timeout."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        with torch.inference_mode(False):
            w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = w
    return w


def check_device_status(device: torch.device) -> None:
    """Synchronise and raise if any kernel on `device` reported a timeout."""
    lib = _lib.load()
    w = status_word(device)
    code = C.c_int(0)
    _lib.check(lib.ttj_read_status(w.data_ptr(), C.byref(code), _stream(device)), "device status")


def _mask_u8(mask: Optional[torch.Tensor], b: int, s: int) -> Optional[torch.Tensor]:
    if mask is None:
        return None
    if mask.shape != (b, s):
        raise RuntimeError(f"valid_token_mask must be [B,S]=({b},{s}), got {tuple(mask.shape)}")
    mask = _cuda(mask, "valid_token_mask")
    if mask.dtype == torch.bool:
        return mask.view(torch.uint8)
    return (mask != 0).view(torch.uint8)


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor,
           residual: Optional[torch.Tensor] = None,
           row_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x w^T + b (+ residual with masked rows keeping only the residual)."""
    lib = _lib.load()
    x, w, bias = _cuda(x, "x"), _cuda(w, "w"), _cuda(bias, "bias")
    dt = _dtype_code(x)
    if w.dtype != x.dtype or bias.dtype != x.dtype:
        raise RuntimeError("x, w and bias must share one dtype")
    k = x.shape[-1]
    m = x.numel() // k
    n = w.shape[0]
    if residual is not None:
        residual = _cuda(residual, "residual")
        if residual.dtype != x.dtype or residual.numel() != m * n:
            raise RuntimeError("residual must match the output's dtype and shape")
    rm = None
    if row_mask is not None:
        rm = _cuda(row_mask.reshape(-1), "row_mask")
        rm = rm.view(torch.uint8) if rm.dtype == torch.bool else (rm != 0).view(torch.uint8)
    y = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    rc = lib.ttj_linear_fwd(x.data_ptr(), w.data_ptr(), bias.data_ptr(), _ptr(residual), _ptr(rm),
                            y.data_ptr(), m, n, k, dt, status_word(x.device).data_ptr(),
                            _stream(x.device))
    _lib.check(rc, "ttj_linear_fwd")
    return y


def linear_kchunked(x_chunks: torch.Tensor, w: torch.Tensor, bias: torch.Tensor,
                    residual: Optional[torch.Tensor] = None,
                    row_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[m, :] = sum_c x_chunks[c, m, :] . w[:, c*kc:(c+1)*kc]^T + bias (+ residual):
    the linear layer on an input stored K-chunk-major [K/kc, M, kc]."""
    lib = _lib.load()
    x_chunks, w, bias = _cuda(x_chunks, "x_chunks"), _cuda(w, "w"), _cuda(bias, "bias")
    dt = _dtype_code(x_chunks)
    nck, m, kc = x_chunks.shape
    n, k = w.shape
    if nck * kc != k:
        raise RuntimeError("x_chunks chunks * chunk width must equal w's input features")
    if residual is not None:
        residual = _cuda(residual, "residual")
    rm = None
    if row_mask is not None:
        rm = _cuda(row_mask.reshape(-1), "row_mask")
        rm = rm.view(torch.uint8) if rm.dtype == torch.bool else (rm != 0).view(torch.uint8)
    y = torch.empty(m, n, dtype=x_chunks.dtype, device=x_chunks.device)
    rc = lib.ttj_linear_kchunked_fwd(x_chunks.data_ptr(), kc, w.data_ptr(), bias.data_ptr(),
                                     _ptr(residual), _ptr(rm), y.data_ptr(), m, n, k, dt,
                                     status_word(x_chunks.device).data_ptr(), _stream(x_chunks.device))
    _lib.check(rc, "ttj_linear_kchunked_fwd")
    return y


def qkv_proj(x: torch.Tensor, w_qkv: torch.Tensor, b_qkv: torch.Tensor) -> torch.Tensor:
    """[B,S,D] -> packed [B,S,3D] (q | k | v)."""
    lib = _lib.load()
    x = _cuda(x, "x")
    dt = _dtype_code(x)
    B, S, D = x.shape
    qkv = torch.empty(B, S, 3 * D, dtype=x.dtype, device=x.device)
    rc = lib.ttj_qkv_proj_fwd(x.data_ptr(), _cuda(w_qkv, "w_qkv").data_ptr(),
                              _cuda(b_qkv, "b_qkv").data_ptr(), qkv.data_ptr(), B * S, D, dt,
                              status_word(x.device).data_ptr(), _stream(x.device))
    _lib.check(rc, "ttj_qkv_proj_fwd")
    return qkv


def flash_attn(qkv: torch.Tensor, num_heads: int, causal: bool,
               key_mask: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Packed [B,S,3D] -> context [B,S,D] (heads merged), optionally into ``out``."""
    lib = _lib.load()
    qkv = _cuda(qkv, "qkv")
    dt = _dtype_code(qkv)
    B, S, D3 = qkv.shape
    D = D3 // 3
    km = _mask_u8(key_mask, B, S)
    if out is None:
        ctx = torch.empty(B, S, D, dtype=qkv.dtype, device=qkv.device)
    else:
        if out.shape != (B, S, D) or out.dtype != qkv.dtype or not out.is_contiguous():
            raise RuntimeError("out must be a contiguous [B,S,D] tensor of qkv's dtype")
        ctx = out
    rc = lib.ttj_flash_attn_fwd(qkv.data_ptr(), _ptr(km), ctx.data_ptr(), B, S, num_heads,
                                D // num_heads, int(bool(causal)), dt,
                                status_word(qkv.device).data_ptr(), _stream(qkv.device))
    _lib.check(rc, "ttj_flash_attn_fwd")
    return ctx


def attn_layer(x: torch.Tensor, w_qkv: torch.Tensor, b_qkv: torch.Tensor, w_o: torch.Tensor,
               b_o: torch.Tensor, num_heads: int, causal: bool,
               valid_token_mask: Optional[torch.Tensor] = None,
               residual: Optional[torch.Tensor] = None, add_residual: bool = True,
               out: Optional[torch.Tensor] = None,
               workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = residual + attention(x); residual defaults to x (the attention
    layer); ``add_residual=False`` returns the attention output alone."""
    lib = _lib.load()
    x = _cuda(x, "x")
    dt = _dtype_code(x)
    B, S, D = x.shape
    for t, n in ((w_qkv, "w_qkv"), (b_qkv, "b_qkv"), (w_o, "w_o"), (b_o, "b_o")):
        if t.dtype != x.dtype or t.device != x.device:
            raise RuntimeError(f"{n} must be {x.dtype} on {x.device}")
    if add_residual:
        residual = x if residual is None else _cuda(residual, "residual")
        if residual.shape != x.shape or residual.dtype != x.dtype:
            raise RuntimeError("residual must match x's shape and dtype")
    else:
        residual = None
    km = _mask_u8(valid_token_mask, B, S)
    if out is None:
        out = torch.empty_like(x)
    need = lib.ttj_attn_layer_workspace_size(B, S, D, dt)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    a = _lib.AttnLayerArgs(
        x=x.data_ptr(), w_qkv=_cuda(w_qkv, "w_qkv").data_ptr(), b_qkv=_cuda(b_qkv, "b_qkv").data_ptr(),
        w_o=_cuda(w_o, "w_o").data_ptr(), b_o=_cuda(b_o, "b_o").data_ptr(),
        valid_token_mask=_ptr(km), residual=_ptr(residual), out=out.data_ptr(),
        workspace=workspace.data_ptr(), workspace_bytes=workspace.numel(),
        status=status_word(x.device).data_ptr(), batch=B, seq_len=S, d_model=D,
        num_heads=num_heads, causal=int(bool(causal)), dtype=dt)
    _lib.check(lib.ttj_attn_layer_fwd(C.byref(a), _stream(x.device)), "ttj_attn_layer_fwd")
    return out


# ------------------------------------------------------- transformer block

def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float,
              row_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """nn.LayerNorm over the last dimension (fp32 arithmetic); rows whose mask
    entry is False come out as zeros.  fp16, bf16 or fp32 (d <= 4096) rows."""
    lib = _lib.load()
    x = _cuda(x, "x")
    dt = _lib.TTJ_F32 if x.dtype == torch.float32 else _dtype_code(x)
    d = x.shape[-1]
    rows = x.numel() // d
    if weight.dtype != x.dtype or bias.dtype != x.dtype:
        raise RuntimeError("weight and bias must share x's dtype")
    rm = None
    if row_mask is not None:
        rm = _cuda(row_mask.reshape(-1), "row_mask")
        if rm.numel() != rows:
            raise RuntimeError("row_mask must have one entry per row")
        rm = rm.view(torch.uint8) if rm.dtype == torch.bool else (rm != 0).view(torch.uint8)
    y = torch.empty_like(x)
    rc = lib.ttj_layernorm_fwd(x.data_ptr(), _cuda(weight, "weight").data_ptr(),
                               _cuda(bias, "bias").data_ptr(), _ptr(rm), y.data_ptr(), rows, d,
                               float(eps), dt, _stream(x.device))
    _lib.check(rc, "ttj_layernorm_fwd")
    return y


def linear_gelu(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """gelu(x w^T + b) with the exact (erf) GELU, one GEMM launch."""
    lib = _lib.load()
    x, w, bias = _cuda(x, "x"), _cuda(w, "w"), _cuda(bias, "bias")
    dt = _dtype_code(x)
    if w.dtype != x.dtype or bias.dtype != x.dtype:
        raise RuntimeError("x, w and bias must share one dtype")
    k = x.shape[-1]
    m = x.numel() // k
    n = w.shape[0]
    y = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    rc = lib.ttj_linear_gelu_fwd(x.data_ptr(), w.data_ptr(), bias.data_ptr(), y.data_ptr(), m, n, k, dt,
                                 status_word(x.device).data_ptr(), _stream(x.device))
    _lib.check(rc, "ttj_linear_gelu_fwd")
    return y


BLOCK_PARAMS = ("ln1_w", "ln1_b", "w_qkv", "b_qkv", "w_o", "b_o", "ln2_w", "ln2_b",
                "w_in", "b_in", "w_out", "b_out")
# An fp32 block (fp32 residual stream) keeps these in fp32 and the rest in fp16
# (ttj_transformer_block_fwd with TTJ_F32).
BLOCK_F32_STREAM_PARAMS = ("ln1_w", "ln1_b", "b_o", "ln2_w", "ln2_b", "b_out")


def block_param_dtype(name: str, x_dtype: torch.dtype) -> torch.dtype:
    """dtype the block kernels expect for parameter `name` given the input dtype."""
    if x_dtype == torch.float32:
        return torch.float32 if name in BLOCK_F32_STREAM_PARAMS else torch.float16
    return x_dtype


def transformer_block(x: torch.Tensor, params: Dict[str, torch.Tensor], num_heads: int,
                      causal: bool, eps1: float, eps2: float,
                      valid_token_mask: Optional[torch.Tensor] = None,
                      out: Optional[torch.Tensor] = None,
                      workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One pre-norm block (BaselineTransformerBlock.forward) in seven launches;
    ``params`` holds the tensors named in BLOCK_PARAMS (w_qkv packed q|k|v) in
    the dtypes of ``block_param_dtype``: x's dtype for fp16 / bf16 blocks; for
    fp32 x an fp32 residual stream with fp16 tensor-core operands."""
    lib = _lib.load()
    x = _cuda(x, "x")
    dt = _lib.TTJ_F32 if x.dtype == torch.float32 else _dtype_code(x)
    if x.dim() != 3:
        raise RuntimeError(f"x must be [B,S,D], got {tuple(x.shape)}")
    B, S, D = x.shape
    ptrs = {}
    for name in BLOCK_PARAMS:
        t = params[name]
        want = block_param_dtype(name, x.dtype)
        if t.dtype != want or t.device != x.device:
            raise RuntimeError(f"{name} must be {want} on {x.device}")
        ptrs[name] = _cuda(t, name).data_ptr()
    F = params["w_in"].shape[0]
    if params["w_in"].shape != (F, D) or params["w_out"].shape != (D, F) or params["w_qkv"].shape != (3 * D, D):
        raise RuntimeError("block weights do not match d_model / ffn_dim")
    km = _mask_u8(valid_token_mask, B, S)
    if out is None:
        out = torch.empty_like(x)
    need = lib.ttj_block_workspace_size(B, S, D, F, dt)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    a = _lib.BlockArgs(x=x.data_ptr(), valid_token_mask=_ptr(km), out=out.data_ptr(),
                       workspace=workspace.data_ptr(), workspace_bytes=workspace.numel(),
                       status=status_word(x.device).data_ptr(), batch=B, seq_len=S, d_model=D,
                       num_heads=num_heads, ffn_dim=F, eps1=float(eps1), eps2=float(eps2),
                       causal=int(bool(causal)), dtype=dt, **ptrs)
    _lib.check(lib.ttj_transformer_block_fwd(C.byref(a), _stream(x.device)), "ttj_transformer_block_fwd")
    return out


# ---------------------------------------------------------------------- int8

def int8_quant_rows(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """[..., K] fp16/bf16 -> (int8 [..., K], fp32 scale [rows])."""
    lib = _lib.load()
    x = _cuda(x, "x")
    dt = _dtype_code(x)
    k = x.shape[-1]
    rows = x.numel() // k
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(rows, dtype=torch.float32, device=x.device)
    _lib.check(lib.ttj_int8_quant_rows(x.data_ptr(), q.data_ptr(), s.data_ptr(), rows, k, dt,
                                       _stream(x.device)), "ttj_int8_quant_rows")
    return q, s


def int8_gemm_s32(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Raw int32 accumulators a[M,K] . w[N,K]^T."""
    lib = _lib.load()
    a, w = _cuda(a, "a"), _cuda(w, "w")
    if a.dtype != torch.int8 or w.dtype != torch.int8:
        raise RuntimeError("int8_gemm_s32 takes int8 operands")
    m, k = a.shape
    n = w.shape[0]
    acc = torch.empty(m, n, dtype=torch.int32, device=a.device)
    _lib.check(lib.ttj_int8_gemm_s32(a.data_ptr(), w.data_ptr(), acc.data_ptr(), m, n, k,
                                     status_word(a.device).data_ptr(), _stream(a.device)),
               "ttj_int8_gemm_s32")
    return acc


def int8_linear(a: torch.Tensor, s_a: torch.Tensor, w: torch.Tensor, s_w: torch.Tensor,
                bias: torch.Tensor, out_dtype: torch.dtype,
                residual: Optional[torch.Tensor] = None,
                row_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Dequantising int8 GEMM: acc * (s_a * s_w) + bias (+ residual)."""
    lib = _lib.load()
    a, w = _cuda(a, "a"), _cuda(w, "w")
    m, k = a.shape
    n = w.shape[0]
    dt = _DTYPES[out_dtype]
    y = torch.empty(m, n, dtype=out_dtype, device=a.device)
    rm = None
    if row_mask is not None:
        rm = _cuda(row_mask.reshape(-1), "row_mask")
        rm = rm.view(torch.uint8) if rm.dtype == torch.bool else (rm != 0).view(torch.uint8)
    if residual is not None:
        residual = _cuda(residual, "residual")
    _lib.check(lib.ttj_int8_linear_fwd(a.data_ptr(), _cuda(s_a, "s_a").data_ptr(), w.data_ptr(),
                                       _cuda(s_w, "s_w").data_ptr(), _cuda(bias, "bias").data_ptr(),
                                       _ptr(residual), _ptr(rm), y.data_ptr(), m, n, k, dt,
                                       status_word(a.device).data_ptr(), _stream(a.device)),
               "ttj_int8_linear_fwd")
    return y


def int8_attn_layer(x: torch.Tensor, w_qkv8: torch.Tensor, s_qkv: torch.Tensor,
                    b_qkv: torch.Tensor, w_o8: torch.Tensor, s_o: torch.Tensor,
                    b_o: torch.Tensor, num_heads: int, causal: bool,
                    valid_token_mask: Optional[torch.Tensor] = None,
                    residual: Optional[torch.Tensor] = None, add_residual: bool = True,
                    out: Optional[torch.Tensor] = None,
                    workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """W8A8 attention layer (benchmark configuration 3 recipe)."""
    lib = _lib.load()
    x = _cuda(x, "x")
    dt = _dtype_code(x)
    B, S, D = x.shape
    if add_residual:
        residual = x if residual is None else _cuda(residual, "residual")
    else:
        residual = None
    km = _mask_u8(valid_token_mask, B, S)
    if out is None:
        out = torch.empty_like(x)
    need = lib.ttj_int8_attn_layer_workspace_size(B, S, D, dt)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    a = _lib.Int8AttnLayerArgs(
        x=x.data_ptr(), w_qkv=_cuda(w_qkv8, "w_qkv").data_ptr(), s_qkv=_cuda(s_qkv, "s_qkv").data_ptr(),
        b_qkv=_cuda(b_qkv, "b_qkv").data_ptr(), w_o=_cuda(w_o8, "w_o").data_ptr(),
        s_o=_cuda(s_o, "s_o").data_ptr(), b_o=_cuda(b_o, "b_o").data_ptr(),
        valid_token_mask=_ptr(km), residual=_ptr(residual), out=out.data_ptr(),
        workspace=workspace.data_ptr(), workspace_bytes=workspace.numel(),
        status=status_word(x.device).data_ptr(), batch=B, seq_len=S, d_model=D,
        num_heads=num_heads, causal=int(bool(causal)), dtype=dt)
    _lib.check(lib.ttj_int8_attn_layer_fwd(C.byref(a), _stream(x.device)), "ttj_int8_attn_layer_fwd")
    return out


def quantize_weight(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel int8 weight packing (one-time, at weight load):
    s = max|w| / 127 clamped to >= 1e-8, q = round(w / s)
    (Project/kernels/k008_int8_gemm.py:154-158).  Runs as torch ops on the
    weights' device; it is set-up, not part of the timed forward."""
    wf = w.float()
    amax = wf.abs().amax(dim=1)
    # Divide by a tensor, not a Python scalar: CUDA torch turns a scalar
    # divisor into a reciprocal multiply, which is not the recipe's IEEE
    # division and can move the scale by one ulp.
    s = (amax / torch.full_like(amax, 127.0)).clamp(min=1e-8)
    q = torch.round(wf / s[:, None]).to(torch.int8)
    return q.contiguous(), s.contiguous()
