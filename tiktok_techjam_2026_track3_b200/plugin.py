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
reference's) and runs its forward on the sm_100a kernels.

fp16 / bf16 models run each ``BaselineTransformerBlock`` (Ref:134-145) as one
``ttj_transformer_block_fwd`` call: LayerNorm, QKV GEMM, flash attention,
out-proj GEMM with bias + mask + residual, LayerNorm, ffn_in GEMM with bias +
exact GELU, ffn_out GEMM with bias + residual + the block's row zeroing; the
final norm and its masked_fill (Ref:169-171) are one LayerNorm launch.

fp32 models (the benchmark's default dtype) run the attention sublayer with
fp16 tensor-core operands and fp32 accumulation, added to the fp32 residual in
fp32; LayerNorm and the FFN stay the reference's own fp32 torch modules.
Whether that meets the benchmark's tolerance is checked by the GPU tests
against the fp32 reference.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .layer import B200SelfAttention

__all__ = ["make_user_optimized_transformer", "build", "attention_sublayer"]

_CACHE_ATTR = "_ttj_attention"
_BLOCK_ATTR = "_ttj_block"


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


def _block_params(block) -> Dict[str, torch.Tensor]:
    """The block's parameters in the kernels' layout (q|k|v packed), cached and
    rebuilt when any parameter's storage or version changes."""
    from .layer import _version
    att = block.attention
    src = (block.norm1.weight, block.norm1.bias, att.q_proj.weight, att.q_proj.bias,
           att.k_proj.weight, att.k_proj.bias, att.v_proj.weight, att.v_proj.bias,
           att.out_proj.weight, att.out_proj.bias, block.norm2.weight, block.norm2.bias,
           block.ffn_in.weight, block.ffn_in.bias, block.ffn_out.weight, block.ffn_out.bias)
    key = tuple((t.data_ptr(), _version(t), t.dtype) for t in src)
    cached = block.__dict__.get(_BLOCK_ATTR)
    if cached is not None and cached[0] == key:
        return cached[1]
    with torch.no_grad():
        t = [p.detach() for p in src]
        packed = {
            "ln1_w": t[0], "ln1_b": t[1],
            "w_qkv": torch.cat([t[2], t[4], t[6]], 0).contiguous(),
            "b_qkv": torch.cat([t[3], t[5], t[7]], 0).contiguous(),
            "w_o": t[8].contiguous(), "b_o": t[9], "ln2_w": t[10], "ln2_b": t[11],
            "w_in": t[12].contiguous(), "b_in": t[13], "w_out": t[14].contiguous(), "b_out": t[15],
        }
    block.__dict__[_BLOCK_ATTR] = (key, packed)
    return packed


def _block_forward(block, x, mask, causal):
    if x.dtype in (torch.float16, torch.bfloat16):
        return ops.transformer_block(x, _block_params(block), block.attention.num_heads, causal,
                                     block.norm1.eps, block.norm2.eps, mask)
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
            if x.dtype in (torch.float16, torch.bfloat16):
                fn = self.final_norm
                return ops.layernorm(x, fn.weight.detach(), fn.bias.detach(), fn.eps, row_mask=mask)
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
