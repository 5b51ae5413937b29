"""Integer reference for the W8A8 projection recipe (test infrastructure only).

Restates the reference's int8 recipe, ``Project/kernels/k008_int8_gemm.py``
(cited ``K8:<line>``):

* activations: per-token symmetric scale ``max|x| clamped to >= 1e-6, / 127``,
  ``round`` half-to-even, int8 (K8:148-151);
* weights: per-output-channel scale ``max|w| / 127 clamped to >= 1e-8``,
  ``round``, int8 (K8:154-158);
* int32 accumulation of int8 x int8 (``torch._int_mm``, K8:183);
* dequant ``acc * (s_tok * s_ch) + bias`` in fp32 (K8:184-185).

The integer GEMM here is exact (float64 accumulation of int8 products, which
is exact at these sizes, checked to fit int32), so the CUDA int8 GEMM's raw
accumulators are compared bit for bit.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from .attention_ref import LayerWeights, split_heads

__all__ = [
    "int8_attention_layer_ref",
    "int8_linear_ref",
    "int_gemm_ref",
    "quant_rows_ref",
    "quant_weight_ref",
]


def _c127(like: torch.Tensor) -> torch.Tensor:
    """127 as a tensor.  Dividing by a tensor keeps the IEEE division the
    recipe specifies on every device (CUDA torch rewrites division by a Python
    scalar as a reciprocal multiply, which can differ by one ulp)."""
    return torch.full_like(like, 127.0)


def quant_rows_ref(t: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-row (per-token) int8 of an fp32 [N,K] matrix -> (int8 [N,K], scale [N]).
    K8:148-151: clamp the row max before dividing by 127."""
    t = t.float()
    amax = t.abs().amax(dim=-1).clamp(min=1e-6)
    s = amax / _c127(amax)
    q = torch.round(t / s[:, None]).to(torch.int8)
    return q, s


def quant_weight_ref(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel int8 of an (out, in) weight -> (int8 [out,in], scale [out]).
    K8:154-158: divide the row max by 127, then clamp.  The weight stays
    (out, in) row-major here (K-major for the GEMM); K8 transposes it only
    because ``torch._int_mm`` wants [K, N]."""
    w = w.float()
    amax = w.abs().amax(dim=1)
    s = (amax / _c127(amax)).clamp(min=1e-8)
    q = torch.round(w / s[:, None]).to(torch.int8)
    return q, s


def int_gemm_ref(a8: torch.Tensor, w8: torch.Tensor) -> torch.Tensor:
    """Exact int32 ``a8 [M,K] @ w8[N,K]^T`` on the operands' device.

    Accumulates in float64: every product of two int8 values is at most 2^14
    in magnitude and any sum of K < 2^38 of them stays below 2^53, so each
    partial sum is an exactly representable integer and the result equals
    integer arithmetic (``torch._int_mm``, K8:183) bit for bit.  Checks the
    result fits int32."""
    if a8.shape[1] >= 2 ** 38:
        raise ValueError("K too large for exact float64 accumulation")
    acc = a8.to(torch.float64) @ w8.to(torch.float64).T
    if acc.numel():
        assert float(acc.abs().max()) < 2.0 ** 31, "int32 accumulator overflow"
    return acc.to(torch.int32)


def int8_linear_ref(h: torch.Tensor, w8: torch.Tensor, s_w: torch.Tensor,
                    bias: torch.Tensor) -> torch.Tensor:
    """fp32 [N,K] -> fp32 [N,out] through the k008 recipe (K8:181-185)."""
    a8, s_a = quant_rows_ref(h)
    acc = int_gemm_ref(a8, w8.to(h.device)).to(torch.float32)
    return acc * (s_a[:, None] * s_w.float()[None, :]) + bias.float()[None, :]


def int8_attention_layer_ref(x: torch.Tensor, w: LayerWeights, num_heads: int,
                             causal: bool = True,
                             valid_token_mask: Optional[torch.Tensor] = None,
                             round_to: Optional[torch.dtype] = torch.bfloat16
                             ) -> torch.Tensor:
    """``x + attn(x)`` with both projections through the int8 recipe.

    Attention itself is fp32 here.  ``round_to`` rounds the dequantised q/k/v
    and the attention context to that dtype, which is what a kernel that
    stores them in bf16 does, so the checker sees the same quantiser inputs."""
    B, S, D = x.shape
    hd = D // num_heads
    wf = w.to(dtype=torch.float32, device=x.device)
    xf = x.float()
    rnd = (lambda t: t.to(round_to).float()) if round_to is not None else (lambda t: t)
    wqkv = torch.cat([wf.wq, wf.wk, wf.wv], 0)
    bqkv = torch.cat([wf.bq, wf.bk, wf.bv], 0)
    wq8, sq = quant_weight_ref(wqkv)
    wo8, so = quant_weight_ref(wf.wo)
    qkv = rnd(int8_linear_ref(xf.reshape(B * S, D), wq8, sq, bqkv)).view(B, S, 3 * D)
    q, k, v = (split_heads(t, num_heads) for t in qkv.split(D, dim=-1))
    scores = torch.matmul(q, k.transpose(-2, -1)) * hd ** -0.5
    if causal:
        scores = scores.masked_fill(torch.ones(S, S, dtype=torch.bool, device=x.device).triu(1),
                                    float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    ctx = torch.matmul(torch.softmax(scores, -1), v).transpose(1, 2).reshape(B * S, D)
    out = int8_linear_ref(rnd(ctx), wo8, so, wf.bo).view(B, S, D)
    if valid_token_mask is not None:
        out = out.masked_fill(~valid_token_mask[..., None], 0)
    return xf + out
