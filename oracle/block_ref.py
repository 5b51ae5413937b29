"""fp32 restatement of the reference's transformer block and model (test
infrastructure only), with the reference's module and parameter names so
state dicts move between them unchanged.

Follows ``torch_transformer_benchmark.py`` (``Ref:<line>``):
``BaselineTransformerBlock`` (Ref:125-145) and ``BaselineTransformer``
(Ref:148-172).  The attention sublayer is ``BaselineSelfAttentionRef``, whose
forward is ``attention_layer_ref`` without the residual (Ref:85-122).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention_ref import LayerWeights, attention_layer_ref

__all__ = ["TransformerConfigRef", "BaselineSelfAttentionRef", "BaselineTransformerBlockRef",
           "BaselineTransformerRef", "streamed_model_ref"]


@dataclass(frozen=True)
class TransformerConfigRef:
    """Fields of the reference's TransformerConfig (Ref:29-37)."""
    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool


def _attention_in_dtype(x, m, num_heads, valid_token_mask, causal):
    """Ref:85-122 evaluated in x's dtype, op for op as the reference does in a
    16-bit run (16-bit matmuls, fp32 softmax cast back, 16-bit out-proj)."""
    B, S, D = x.shape
    hd = D // num_heads
    def heads(t):
        return t.view(B, S, num_heads, hd).transpose(1, 2).contiguous()
    q, k, v = heads(m.q_proj(x)), heads(m.k_proj(x)), heads(m.v_proj(x))
    scores = torch.matmul(q, k.transpose(-2, -1)) * hd ** -0.5
    if causal:
        scores = scores.masked_fill(torch.ones(S, S, device=x.device, dtype=torch.bool).triu(1), float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)
    ctx = torch.matmul(probs, v).transpose(1, 2).contiguous().view(B, S, D)
    out = m.out_proj(ctx)
    if valid_token_mask is not None:
        out = out.masked_fill(~valid_token_mask[..., None], 0)
    return out


class BaselineSelfAttentionRef(nn.Module):
    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)

    def forward(self, x, valid_token_mask=None, causal=False, in_dtype=False):
        if in_dtype:
            return _attention_in_dtype(x, self, self.num_heads, valid_token_mask, causal)
        w = LayerWeights(self.q_proj.weight, self.q_proj.bias, self.k_proj.weight, self.k_proj.bias,
                         self.v_proj.weight, self.v_proj.bias, self.out_proj.weight, self.out_proj.bias)
        return attention_layer_ref(x, w, self.num_heads, valid_token_mask, causal, residual=False)


class BaselineTransformerBlockRef(nn.Module):
    """Pre-norm block: x + attn(norm1(x)); x + ffn_out(gelu_exact(ffn_in(norm2(x))));
    invalid rows zeroed (Ref:125-145)."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = BaselineSelfAttentionRef(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def forward(self, x, valid_token_mask, causal, in_dtype=False):
        if in_dtype:  # the reference's own low-precision run (Ref:134-145 in x's dtype)
            x = x + self.attention(self.norm1(x), valid_token_mask, causal, in_dtype=True)
            x = x + self.ffn_out(F.gelu(self.ffn_in(self.norm2(x)), approximate="none"))
            if valid_token_mask is not None:
                x = x.masked_fill(~valid_token_mask[..., None], 0)
            return x
        x = x.float()
        x = x + self.attention(F.layer_norm(x, x.shape[-1:], self.norm1.weight.float(), self.norm1.bias.float()),
                               valid_token_mask, causal)
        h = F.layer_norm(x, x.shape[-1:], self.norm2.weight.float(), self.norm2.bias.float())
        h = F.gelu(F.linear(h, self.ffn_in.weight.float(), self.ffn_in.bias.float()), approximate="none")
        x = x + F.linear(h, self.ffn_out.weight.float(), self.ffn_out.bias.float())
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


class BaselineTransformerRef(nn.Module):
    """Stack of blocks, final LayerNorm, masked rows zeroed (Ref:148-172), in fp32."""

    def __init__(self, config) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList([BaselineTransformerBlockRef(config.d_model, config.num_heads,
                                                                 config.ffn_dim)
                                     for _ in range(config.num_layers)])
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x, valid_token_mask: Optional[torch.Tensor] = None, in_dtype: bool = False):
        """fp32 by default; ``in_dtype=True`` keeps every op in the parameters'
        dtype, as the reference model does when the benchmark runs in fp16/bf16."""
        if in_dtype:
            for layer in self.layers:
                x = layer(x, valid_token_mask, self.config.causal, in_dtype=True)
            x = self.final_norm(x)
            if valid_token_mask is not None:
                x = x.masked_fill(~valid_token_mask[..., None], 0)
            return x
        for layer in self.layers:
            x = layer(x, valid_token_mask, self.config.causal)
        x = F.layer_norm(x.float(), x.shape[-1:], self.final_norm.weight.float(), self.final_norm.bias.float())
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


def _streamed_heads_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                              causal: bool, key_mask: Optional[torch.Tensor],
                              q_chunk: int, k_chunk: int) -> torch.Tensor:
    """softmax(q k^T * scale + masks) v for one batch row, all heads at once
    ([H,S,hd] each), in fp32 over (query chunk x key chunk) blocks with a
    running max and sum: the S x S table never exists.  Causal query chunks
    stop at their last row's key.  Rows that see no key (possible only with a
    key mask) come out as zeros."""
    H, S, hd = q.shape
    out = torch.empty_like(q)
    for qs in range(0, S, q_chunk):
        qe = min(qs + q_chunk, S)
        run_max = torch.full((H, qe - qs), float("-inf"), device=q.device)
        run_sum = torch.zeros(H, qe - qs, device=q.device)
        acc = torch.zeros(H, qe - qs, hd, device=q.device)
        qidx = torch.arange(qs, qe, device=q.device)
        for ks in range(0, qe if causal else S, k_chunk):
            ke = min(ks + k_chunk, qe if causal else S)
            s = torch.matmul(q[:, qs:qe], k[:, ks:ke].transpose(1, 2)).mul_(scale)
            kidx = torch.arange(ks, ke, device=q.device)
            if causal and ke - 1 > qs:
                s.masked_fill_((kidx[None, :] > qidx[:, None])[None], float("-inf"))
            if key_mask is not None:
                s.masked_fill_(~key_mask[ks:ke][None, None, :], float("-inf"))
            new_max = torch.maximum(run_max, s.amax(dim=2))
            safe = torch.where(torch.isinf(new_max), torch.zeros_like(new_max), new_max)
            alpha = torch.exp(run_max - safe)
            p = s.sub_(safe[..., None]).exp_()
            run_sum = run_sum * alpha + p.sum(dim=2)
            acc = acc * alpha[..., None] + torch.matmul(p, v[:, ks:ke])
            run_max = new_max
            del s, p
        out[:, qs:qe] = acc / torch.where(run_sum > 0, run_sum, torch.ones_like(run_sum))[..., None]
    return out


def streamed_model_ref(model: "BaselineTransformerRef", x: torch.Tensor,
                       valid_token_mask: Optional[torch.Tensor] = None,
                       q_chunk: int = 4096, k_chunk: int = 16384) -> torch.Tensor:
    """``BaselineTransformer.forward`` (Ref:148-172, blocks Ref:125-145) in fp32
    for sequences whose score table cannot be held (the reference's official
    shape 14, S = 100000): the model's own LayerNorms, projections, exact-erf
    FFN and final norm, with each attention evaluated over (query chunk x key
    chunk) blocks with a running max and sum.  That is the behaviour of the
    reference's long-context checker (Project/tools/shape14_eval.py:201-254,
    which swaps ``attention.forward`` for a streamed version); here all heads
    of a batch row go through each block together.  Batch rows are evaluated
    one at a time, on x's device; returns fp32 [B,S,D]."""
    cfg = model.config
    B, S, D = x.shape
    H = cfg.num_heads
    hd = D // H
    out = torch.empty(B, S, D, device=x.device)

    def lin(t, m):
        return F.linear(t, m.weight.float(), m.bias.float())

    def norm(t, m):
        return F.layer_norm(t, (D,), m.weight.float(), m.bias.float(), m.eps)

    for b in range(B):
        h = x[b].float()
        km = None if valid_token_mask is None else valid_token_mask[b].to(x.device)
        for layer in model.layers:
            att = layer.attention
            a = norm(h, layer.norm1)
            q, k, v = (lin(a, m).view(S, H, hd).transpose(0, 1).contiguous()
                       for m in (att.q_proj, att.k_proj, att.v_proj))
            ctx = _streamed_heads_attention(q, k, v, hd ** -0.5, cfg.causal, km, q_chunk, k_chunk)
            del q, k, v
            o = lin(ctx.transpose(0, 1).reshape(S, D), att.out_proj)           # Ref:113-118
            if km is not None:
                o = o.masked_fill(~km[:, None], 0)                              # Ref:120-121
            h = h + o                                                           # Ref:140
            f = lin(F.gelu(lin(norm(h, layer.norm2), layer.ffn_in), approximate="none"), layer.ffn_out)
            h = h + f                                                           # Ref:141-142
            if km is not None:
                h = h.masked_fill(~km[:, None], 0)                              # Ref:143-144
        h = norm(h, model.final_norm)                                           # Ref:168
        if km is not None:
            h = h.masked_fill(~km[:, None], 0)                                  # Ref:170-171
        out[b] = h
    return out
