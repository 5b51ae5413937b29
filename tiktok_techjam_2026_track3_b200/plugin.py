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

Every ``BaselineTransformerBlock`` (Ref:134-145) is one
``ttj_transformer_block_fwd`` call: LayerNorm, QKV GEMM, flash attention,
out-proj GEMM with bias + mask + residual, LayerNorm, ffn_in GEMM with bias +
exact GELU, ffn_out GEMM with bias + residual + the block's row zeroing; the
final norm and its masked_fill (Ref:169-171) are one LayerNorm launch.
fp16 / bf16 models run in their own dtype.  fp32 models (the benchmark's
default dtype) keep the residual stream, the LayerNorm parameters and the
residual-side biases in fp32 and run every GEMM and the attention on fp16
copies of the weights (fp32 accumulation inside every kernel): the LayerNorm
kernels read the fp32 stream and write fp16 operands, the out-proj and ffn_out
epilogues add in fp32 and write the fp32 stream.  The reference's own optimised
route runs fp32 models on fp16 weights too (Project/submission/dispatcher_region.py:760-801),
with an fp16 stream; measured on the official shapes, an fp16 stream misses
the benchmark tolerance on a few elements, the fp32 stream meets it (the GPU
tests hold every shape to it against the fp32 reference).

Repeated calls with the same input shape, dtype, mask presence and weights are
replayed from a CUDA graph captured on the second such call (the reference's
route does the same, dispatcher_region.py:1220-1260): the input (and mask) are
copied into the graph's static buffers and the output is returned as a fresh
copy, never the graph's own buffer.  Only launch-bound sizes (at most 2^24
activation elements) are captured; larger calls run eagerly, where launch
overhead is negligible.  ``model.ttj_cuda_graphs = False`` turns capture off.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn

from . import ops
from .layer import B200SelfAttention, _version

__all__ = ["make_user_optimized_transformer", "build", "attention_sublayer", "block_forward"]

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


_GRAPH_MAX_ELEMENTS = 1 << 24


def _check_dtype(dtype: torch.dtype) -> None:
    if dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise RuntimeError(f"unsupported dtype {dtype}: the sm_100a kernels take float32, float16 or bfloat16 models")


def _block_params(block, dtype: torch.dtype) -> Dict[str, torch.Tensor]:
    """The block's parameters in the kernels' layout (q|k|v packed) and the
    dtypes ``ops.block_param_dtype`` gives for a `dtype` input, cached and
    rebuilt when any parameter's storage or version changes."""
    att = block.attention
    src = (block.norm1.weight, block.norm1.bias, att.q_proj.weight, att.q_proj.bias,
           att.k_proj.weight, att.k_proj.bias, att.v_proj.weight, att.v_proj.bias,
           att.out_proj.weight, att.out_proj.bias, block.norm2.weight, block.norm2.bias,
           block.ffn_in.weight, block.ffn_in.bias, block.ffn_out.weight, block.ffn_out.bias)
    key = (dtype,) + tuple((t.data_ptr(), _version(t), t.dtype) for t in src)
    cached = block.__dict__.get(_BLOCK_ATTR)
    if cached is not None and cached[0] == key:
        return cached[1]
    with torch.no_grad():
        t = [p.detach() for p in src]
        packed = {
            "ln1_w": t[0], "ln1_b": t[1],
            "w_qkv": torch.cat([t[2], t[4], t[6]], 0), "b_qkv": torch.cat([t[3], t[5], t[7]], 0),
            "w_o": t[8], "b_o": t[9], "ln2_w": t[10], "ln2_b": t[11],
            "w_in": t[12], "b_in": t[13], "w_out": t[14], "b_out": t[15],
        }
        packed = {k: v.to(ops.block_param_dtype(k, dtype)).contiguous() for k, v in packed.items()}
    block.__dict__[_BLOCK_ATTR] = (key, packed)
    return packed


def _final_norm_params(model, dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    fn = model.final_norm
    key = (dtype, fn.weight.data_ptr(), _version(fn.weight), fn.bias.data_ptr(), _version(fn.bias))
    cached = model.__dict__.get("_ttj_final_norm")
    if cached is not None and cached[0] == key:
        return cached[1]
    with torch.no_grad():
        wb = (fn.weight.detach().to(dtype).contiguous(), fn.bias.detach().to(dtype).contiguous())
    model.__dict__["_ttj_final_norm"] = (key, wb)
    return wb


def block_forward(block, x: torch.Tensor, mask: Optional[torch.Tensor], causal: bool) -> torch.Tensor:
    """One BaselineTransformerBlock.forward (Ref:134-145) as one
    ttj_transformer_block_fwd call.  fp16 / bf16 x: the block in that dtype;
    fp32 x: an fp32 residual stream with fp16 tensor-core operands (the
    block's parameters are converted once and cached)."""
    return ops.transformer_block(x, _block_params(block, x.dtype), block.attention.num_heads, causal,
                                 block.norm1.eps, block.norm2.eps, mask)


def _model_forward(model, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
    """Blocks + final norm on the kernels (residual stream in x's dtype)."""
    _check_dtype(x.dtype)
    h = x
    for layer in model.layers:
        h = block_forward(layer, h, mask, model.config.causal)
    w, b = _final_norm_params(model, x.dtype)
    return ops.layernorm(h, w, b, model.final_norm.eps, row_mask=mask)


def _weights_key(model):
    return tuple((p.data_ptr(), _version(p), p.dtype) for p in model.parameters())


class _GraphRunner:
    """One captured forward per model: (shape, dtype, device, mask presence,
    weights) must match for a replay; a new key runs eagerly once and is
    captured on its second call."""

    def __init__(self) -> None:
        self.key = None
        self.pending = None
        self.graph = None
        self.static_x = None
        self.static_mask = None
        self.static_out = None

    def __call__(self, model, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        key = (tuple(x.shape), x.dtype, x.device, None if mask is None else tuple(mask.shape),
               _weights_key(model))
        if self.graph is not None and key == self.key:
            self.static_x.copy_(x)
            if mask is not None:
                self.static_mask.copy_(mask)
            self.graph.replay()
            return self.static_out.clone()
        if key != self.pending:
            self.pending = key
            return _model_forward(model, x, mask)   # first call: eager (packs weights)
        # second call with this key: capture
        self.graph = None
        self.static_x = x.clone()
        self.static_mask = None if mask is None else mask.clone()
        graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(x.device)
        with torch.cuda.graph(graph):
            self.static_out = _model_forward(model, self.static_x, self.static_mask)
        self.graph, self.key, self.pending = graph, key, None
        self.graph.replay()
        return self.static_out.clone()


def make_user_optimized_transformer(base_cls):
    """Subclass of the reference's BaselineTransformer on the sm_100a kernels."""

    class UserOptimizedTransformer(base_cls):
        ttj_cuda_graphs = True

        def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
            if not x.is_cuda:
                raise RuntimeError(f"x must be a CUDA tensor (got {x.device}); there is no CPU path")
            mask = None if valid_token_mask is None else valid_token_mask.to(torch.bool)
            if (self.ttj_cuda_graphs and x.is_contiguous() and x.numel() <= _GRAPH_MAX_ELEMENTS
                    and not torch.cuda.is_current_stream_capturing()):
                runner = self.__dict__.get("_ttj_graph_runner")
                if runner is None:
                    runner = _GraphRunner()
                    self.__dict__["_ttj_graph_runner"] = runner
                return runner(self, x.contiguous(), mask)
            return _model_forward(self, x, mask)

    UserOptimizedTransformer.__name__ = "UserOptimizedTransformer"
    UserOptimizedTransformer.__qualname__ = "UserOptimizedTransformer"
    return UserOptimizedTransformer


def build(otb, config) -> nn.Module:
    """Harness plugin entry (Project/harness/candidate_worker.py:275-294): ``otb`` is
    the imported benchmark script, ``config`` its TransformerConfig."""
    return make_user_optimized_transformer(otb.BaselineTransformer)(config)
