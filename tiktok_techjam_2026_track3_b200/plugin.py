"""Drop-in for the reference benchmark's model slot.

The reference benchmark (torch_transformer_benchmark.py) compares
``BaselineTransformer`` with a ``UserOptimizedTransformer`` that must keep the
forward signature ``forward(x, valid_token_mask=None) -> [B,S,D]`` and
compatible parameter names (torch_transformer_benchmark.py:175-200); its
harness loads candidates through a module-level ``build(otb, config)`` where
``otb`` is the imported benchmark script
(Project/harness/candidate_worker.py:275-294).

``make_user_optimized_transformer(base_cls)`` subclasses the reference's own
``BaselineTransformer`` (so the module tree and state-dict keys are the
reference's) and replaces, in every block, ``x + attention(norm1(x))``
(torch_transformer_benchmark.py:140) with the sm_100a attention layer: QKV GEMM,
flash attention, out-proj GEMM whose epilogue adds the bias, zeroes invalid
rows and adds the pre-norm residual.  LayerNorm, the exact-erf GELU FFN and the
final norm run as the reference's own torch modules.

Inputs in fp16 / bf16 run the kernels in that dtype.  fp32 inputs (the
benchmark's default dtype) run the attention sublayer with fp16 tensor-core
operands and fp32 accumulation; its output is added to the fp32 residual in
fp32.  Whether that meets the benchmark's tolerance is checked by the GPU tests
against the fp32 reference.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layer import B200SelfAttention

__all__ = ["make_user_optimized_transformer", "build", "attention_sublayer"]

_CACHE_ATTR = "_ttj_attention"


def attention_sublayer(block: nn.Module) -> B200SelfAttention:
    """A B200SelfAttention sharing ``block.attention``'s four Linear modules
    (no copy; not registered as a submodule, so the state dict is unchanged)."""
    cached = block.__dict__.get(_CACHE_ATTR)
    src = block.attention
    if cached is not None and cached.q_proj is src.q_proj:
        return cached
    attn = B200SelfAttention.__new__(B200SelfAttention)
    nn.Module.__init__(attn)
    attn.d_model, attn.num_heads = src.d_model, src.num_heads
    attn.head_dim = src.d_model // src.num_heads
    attn.scale = attn.head_dim ** -0.5
    attn.quant = None
    attn.q_proj, attn.k_proj, attn.v_proj, attn.out_proj = src.q_proj, src.k_proj, src.v_proj, src.out_proj
    attn._pack_key = None
    attn._packed = None
    block.__dict__[_CACHE_ATTR] = attn
    return attn


def _attention_residual(block, x: torch.Tensor, mask: Optional[torch.Tensor], causal: bool) -> torch.Tensor:
    attn = attention_sublayer(block)
    h = block.norm1(x)
    if x.dtype in (torch.float16, torch.bfloat16):
        return attn.forward_residual(h, x, mask, causal)
    if x.dtype != torch.float32:
        raise RuntimeError(f"unsupported dtype {x.dtype}")
    # fp32 model: fp16 operands on the tensor cores, fp32 accumulate, fp32 residual.
    half = _half_view(attn)
    return x + half.forward(h.to(torch.float16), mask, causal).float()


def _half_view(attn: B200SelfAttention) -> B200SelfAttention:
    """An fp16 copy of the projection weights for fp32 models (rebuilt when the
    fp32 weights change)."""
    from .layer import _version
    key = tuple((p.data_ptr(), _version(p)) for p in attn._params())
    cached = attn.__dict__.get("_ttj_half")
    if cached is not None and cached[0] == key:
        return cached[1]
    with torch.inference_mode(False), torch.no_grad():
        half = B200SelfAttention(attn.d_model, attn.num_heads).to(device=attn.q_proj.weight.device)
        for dst, src in zip(half._params(), attn._params()):
            dst.copy_(src.detach().clone() if src.is_inference() else src)
        half = half.half()
    attn.__dict__["_ttj_half"] = (key, half)
    return half


def _block_forward(block, x, mask, causal):
    x = _attention_residual(block, x, mask, causal)
    x = x + block.ffn_out(F.gelu(block.ffn_in(block.norm2(x)), approximate="none"))
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
    return x


def make_user_optimized_transformer(base_cls):
    """Subclass of the reference's BaselineTransformer with the sm_100a attention."""

    class UserOptimizedTransformer(base_cls):
        def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
            mask = None if valid_token_mask is None else valid_token_mask.to(torch.bool)
            for layer in self.layers:
                x = _block_forward(layer, x, mask, self.config.causal)
            x = self.final_norm(x)
            if mask is not None:
                x = x.masked_fill(~mask[..., None], 0)
            return x

    UserOptimizedTransformer.__name__ = "UserOptimizedTransformer"
    UserOptimizedTransformer.__qualname__ = "UserOptimizedTransformer"
    return UserOptimizedTransformer


def build(otb, config) -> nn.Module:
    """Harness plugin entry (Project/harness/candidate_worker.py:275-294): ``otb`` is
    the imported benchmark script, ``config`` its TransformerConfig."""
    return make_user_optimized_transformer(otb.BaselineTransformer)(config)
