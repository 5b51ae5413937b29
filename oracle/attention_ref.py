"""fp32 restatement of the reference attention layer (test infrastructure only).

Every function here restates the behaviour of the reference benchmark
``torch_transformer_benchmark.py`` (cited below as ``Ref:<line>``) in plain fp32
PyTorch so the CUDA kernels can be checked against it.  Nothing here is shipped
or timed as the product; the product never imports this module.

Device-agnostic: tests run it on the CPU for small cases and, for sampled
stripes of the long-context configurations, in fp32 on the GPU with TF32
disabled (the reference itself enables TF32 on CUDA, Ref:687-688, which is
noisier than the checker should be).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch

__all__ = [
    "AccuracyReport",
    "LayerWeights",
    "attention_layer_ref",
    "attention_layer_rows_ref",
    "attention_layer_streamed_ref",
    "compare_outputs",
    "generate_case",
    "make_weights",
    "split_heads",
    "streamed_attention_ref",
]


@dataclass
class LayerWeights:
    """The four ``nn.Linear(D, D, bias=True)`` of ``BaselineSelfAttention``
    (Ref:72-75), stored as (out, in) row-major weights and (out,) biases."""

    wq: torch.Tensor
    bq: torch.Tensor
    wk: torch.Tensor
    bk: torch.Tensor
    wv: torch.Tensor
    bv: torch.Tensor
    wo: torch.Tensor
    bo: torch.Tensor

    def state_dict(self, prefix: str = "") -> Dict[str, torch.Tensor]:
        """Keys exactly as the reference module names them (Ref:72-75)."""
        return {
            f"{prefix}q_proj.weight": self.wq, f"{prefix}q_proj.bias": self.bq,
            f"{prefix}k_proj.weight": self.wk, f"{prefix}k_proj.bias": self.bk,
            f"{prefix}v_proj.weight": self.wv, f"{prefix}v_proj.bias": self.bv,
            f"{prefix}out_proj.weight": self.wo, f"{prefix}out_proj.bias": self.bo,
        }

    @staticmethod
    def from_state_dict(sd: Dict[str, torch.Tensor], prefix: str = "") -> "LayerWeights":
        g = lambda n: sd[prefix + n]  # noqa: E731
        return LayerWeights(g("q_proj.weight"), g("q_proj.bias"), g("k_proj.weight"),
                            g("k_proj.bias"), g("v_proj.weight"), g("v_proj.bias"),
                            g("out_proj.weight"), g("out_proj.bias"))

    def to(self, *args, **kwargs) -> "LayerWeights":
        return LayerWeights(*(t.to(*args, **kwargs) for t in self.tensors()))

    def tensors(self) -> Tuple[torch.Tensor, ...]:
        return (self.wq, self.bq, self.wk, self.bk, self.wv, self.bv, self.wo, self.bo)


def make_weights(d_model: int, seed: int, std: float = 0.02,
                 dtype: torch.dtype = torch.float32) -> LayerWeights:
    """Seeded N(0, std) weights and biases, the benchmark configurations' choice.

    The reference initialises with ``nn.Linear`` defaults; the benchmark then
    copies one state dict into both models (Ref:203-213), so any seeded values
    work as long as both sides receive the same tensors."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    ts = []
    for _ in range(4):
        ts.append(torch.randn(d_model, d_model, generator=g) * std)
        ts.append(torch.randn(d_model, generator=g) * std)
    return LayerWeights(*ts).to(dtype=dtype)


def generate_case(batch: int, seq_len: int, d_model: int, seed: int,
                  dtype: torch.dtype = torch.float32, padding_ratio: float = 0.0,
                  input_scale: float = 1.0, device: str = "cpu"
                  ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Seeded input and prefix validity mask, as Ref:234-272 generates them.

    Same generator, same draw order (x first, then the per-row lengths), so on
    the CPU it returns bit-identical tensors to the reference's
    ``generate_random_case`` for the same arguments."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    x = torch.randn(batch, seq_len, d_model, generator=gen, device=device, dtype=dtype)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(batch, seq_len, device=device, dtype=torch.bool)
    min_valid = max(1, int(round(seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=seq_len + 1, size=(batch,),
                            generator=gen, device=device)
    mask = torch.arange(seq_len, device=device)[None, :] < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


def split_heads(t: torch.Tensor, num_heads: int) -> torch.Tensor:
    """[B,S,D] -> [B,H,S,hd] (Ref:77-83)."""
    b, s, d = t.shape
    return t.view(b, s, num_heads, d // num_heads).transpose(1, 2).contiguous()


def _linear(t: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.linear(t, w, b)


def attention_layer_ref(x: torch.Tensor, w: LayerWeights, num_heads: int,
                        valid_token_mask: Optional[torch.Tensor] = None,
                        causal: bool = False, residual: bool = True,
                        batch_chunk: Optional[int] = None) -> torch.Tensor:
    """Dense fp32 ``x + BaselineSelfAttention(x)``.

    Follows Ref:85-122 step for step (q/k/v projections, head split, scaled
    scores, causal ``triu(1)`` mask, key-padding mask, fp32 softmax, P·V, head
    merge, out-proj, masked output rows) and the block residual of Ref:140.
    Everything is computed in fp32 whatever ``x.dtype`` is; the result is
    fp32.  ``batch_chunk`` evaluates independent batch rows a slice at a time
    so the [B,H,S,S] score tensor stays bounded (batch rows never interact)."""
    xf = x.float()
    wf = w.to(dtype=torch.float32, device=x.device)
    B, S, D = xf.shape
    if batch_chunk is not None and batch_chunk < B:
        parts = []
        for b0 in range(0, B, batch_chunk):
            m = None if valid_token_mask is None else valid_token_mask[b0:b0 + batch_chunk]
            parts.append(attention_layer_ref(xf[b0:b0 + batch_chunk], wf, num_heads, m,
                                             causal, residual, None))
        return torch.cat(parts, 0)
    hd = D // num_heads
    scale = hd ** -0.5                                           # Ref:70
    q = split_heads(_linear(xf, wf.wq, wf.bq), num_heads)        # Ref:93
    k = split_heads(_linear(xf, wf.wk, wf.bk), num_heads)        # Ref:94
    v = split_heads(_linear(xf, wf.wv, wf.bv), num_heads)        # Ref:95
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale        # Ref:97
    if causal:                                                   # Ref:99-103
        upper = torch.ones(S, S, device=x.device, dtype=torch.bool).triu(1)
        scores = scores.masked_fill(upper, float("-inf"))
    if valid_token_mask is not None:                             # Ref:105-108
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores, dim=-1)                        # Ref:111 (fp32)
    ctx = torch.matmul(probs, v)                                 # Ref:112
    ctx = ctx.transpose(1, 2).contiguous().view(B, S, D)         # Ref:113-117
    out = _linear(ctx, wf.wo, wf.bo)                             # Ref:118
    if valid_token_mask is not None:                             # Ref:120-121
        out = out.masked_fill(~valid_token_mask[..., None], 0)
    return xf + out if residual else out                         # Ref:140


def streamed_attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           scale: float, causal: bool,
                           key_mask: Optional[torch.Tensor] = None,
                           q_rows: Optional[torch.Tensor] = None,
                           k_chunk: int = 8192,
                           probs_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Online-softmax fp32 attention for one (batch, head) slice, no S×S table.

    q: [Sq,hd] (the query rows to evaluate), k/v: [S,hd]; ``q_rows`` gives the
    absolute sequence position of each query row (default ``arange(Sq)``), so
    a sampled stripe of a long sequence can be evaluated on its own.  The
    behaviour follows the reference's long-context checker
    ``Project/tools/shape14_eval.py:201-236``: running max / running sum over
    key chunks, rescaled accumulator, one division at the end.

    ``probs_dtype`` rounds the normalised probabilities to that dtype before
    they multiply v, as the reference's 16-bit run does with
    ``softmax(scores.float()).to(x.dtype)`` (torch_transformer_benchmark.py:111).
    Rounding needs each row's final max and sum first, so that variant makes
    two passes over the keys: the online pass above for max and sum, then
    p = round(exp(s - max) / sum) and the product with v."""
    qf, kf, vf = q.float(), k.float(), v.float()
    Sq = qf.shape[0]
    S = kf.shape[0]
    if q_rows is None:
        q_rows = torch.arange(Sq, device=q.device)
    q_rows = q_rows.to(q.device)
    run_max = torch.full((Sq,), float("-inf"), device=q.device)
    run_sum = torch.zeros(Sq, device=q.device)
    acc = torch.zeros(Sq, vf.shape[1], device=q.device)
    k_end = int(q_rows.max().item()) + 1 if causal else S

    def scores(k0, k1):
        s = (qf @ kf[k0:k1].T) * scale
        kidx = torch.arange(k0, k1, device=q.device)
        if causal:
            s = s.masked_fill(kidx[None, :] > q_rows[:, None], float("-inf"))
        if key_mask is not None:
            s = s.masked_fill(~key_mask[k0:k1][None, :], float("-inf"))
        return s

    for k0 in range(0, k_end, k_chunk):
        k1 = min(k0 + k_chunk, k_end)
        s = scores(k0, k1)
        new_max = torch.maximum(run_max, s.amax(dim=1))
        safe = torch.where(torch.isinf(new_max), torch.zeros_like(new_max), new_max)
        alpha = torch.exp(run_max - safe)
        p = torch.exp(s - safe[:, None])
        run_sum = run_sum * alpha + p.sum(dim=1)
        if probs_dtype is None:
            acc = acc * alpha[:, None] + p @ vf[k0:k1]
        run_max = new_max
    if probs_dtype is None:
        return acc / run_sum[:, None]
    safe = torch.where(torch.isinf(run_max), torch.zeros_like(run_max), run_max)
    for k0 in range(0, k_end, k_chunk):
        k1 = min(k0 + k_chunk, k_end)
        p = torch.exp(scores(k0, k1) - safe[:, None]) / run_sum[:, None]
        acc = acc + p.to(probs_dtype).float() @ vf[k0:k1]
    return acc


def attention_layer_rows_ref(x: torch.Tensor, w: LayerWeights, num_heads: int, causal: bool,
                             batches: Sequence[int], q_rows: torch.Tensor,
                             store_dtypes: Sequence[Optional[torch.dtype]] = (None,),
                             valid_token_mask: Optional[torch.Tensor] = None,
                             k_chunk: int = 16384) -> List[torch.Tensor]:
    """Layer OUTPUT rows ``x + BaselineSelfAttention(x)`` for sampled batch rows
    and query rows, on x's device, one result [len(batches), len(q_rows), D]
    (fp32) per entry of ``store_dtypes``.

    ``None`` evaluates Ref:85-122 + :140 in fp32 throughout: the exact layer for
    the given (already rounded) inputs and weights.  A 16-bit dtype rounds to it
    where the reference's own 16-bit run stores a tensor -- q, k and v after the
    projections (Ref:93-95), the probabilities (Ref:111), the context after the
    head merge (Ref:112-117), the out-proj output (Ref:118) and the residual sum
    (Ref:140) -- except the score matrix, which the reference's 16-bit run also
    rounds but which this checker (like the kernel) keeps in fp32.  Every
    variant shares the fp32 projections, so their differences are exactly the
    roundings.  Only the sampled query rows and the keys they can see are
    computed, which lets sequences of 10^5 - 2.6*10^5 tokens be checked stripe by
    stripe."""
    B, S, D = x.shape
    hd = D // num_heads
    wf = w.to(dtype=torch.float32, device=x.device)
    q_rows = q_rows.to(x.device)
    k_end = int(q_rows.max().item()) + 1 if causal else S
    outs = [torch.empty(len(batches), len(q_rows), D, device=x.device) for _ in store_dtypes]

    def rnd(t, dt):
        return t if dt is None else t.to(dt).float()

    for bi, b in enumerate(batches):
        xb = x[b, :k_end].float()
        km = None if valid_token_mask is None else valid_token_mask[b].to(x.device)
        ctx = [torch.empty(len(q_rows), D, device=x.device) for _ in store_dtypes]
        for h in range(num_heads):
            sl = slice(h * hd, (h + 1) * hd)
            q = _linear(xb[q_rows], wf.wq[sl], wf.bq[sl])
            k = _linear(xb, wf.wk[sl], wf.bk[sl])
            v = _linear(xb, wf.wv[sl], wf.bv[sl])
            for i, dt in enumerate(store_dtypes):
                ctx[i][:, sl] = streamed_attention_ref(rnd(q, dt), rnd(k, dt), rnd(v, dt), hd ** -0.5, causal,
                                                       key_mask=km, q_rows=q_rows, k_chunk=k_chunk,
                                                       probs_dtype=dt)
        for i, dt in enumerate(store_dtypes):
            o = rnd(_linear(rnd(ctx[i], dt), wf.wo, wf.bo), dt)
            if km is not None:
                o = o.masked_fill(~km[q_rows][:, None], 0)
            outs[i][bi] = rnd(xb[q_rows] + o, dt)
    return outs


def attention_layer_streamed_ref(x: torch.Tensor, w: LayerWeights, num_heads: int,
                                 causal: bool, batches: Sequence[int],
                                 heads: Sequence[int], q_rows: torch.Tensor,
                                 k_chunk: int = 8192) -> torch.Tensor:
    """Attention CONTEXT (before out-proj) for sampled (batch, head, rows).

    Returns [len(batches), len(heads), len(q_rows), hd] fp32.  Only the q/k/v
    columns of the sampled heads are projected, so the long-context configs
    (S up to 262144) can be checked stripe by stripe on the GPU box in fp32."""
    B, S, D = x.shape
    hd = D // num_heads
    wf = w.to(dtype=torch.float32, device=x.device)
    out = torch.empty(len(batches), len(heads), len(q_rows), hd, device=x.device)
    for bi, b in enumerate(batches):
        xb = x[b].float()
        for hi, h in enumerate(heads):
            sl = slice(h * hd, (h + 1) * hd)
            qh = _linear(xb[q_rows], wf.wq[sl], wf.bq[sl])
            kh = _linear(xb, wf.wk[sl], wf.bk[sl])
            vh = _linear(xb, wf.wv[sl], wf.bv[sl])
            out[bi, hi] = streamed_attention_ref(qh, kh, vh, hd ** -0.5, causal,
                                                 q_rows=q_rows, k_chunk=k_chunk)
    return out


@dataclass
class AccuracyReport:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    worst_index: Tuple[int, ...]

    def __str__(self) -> str:
        return (f"{'PASS' if self.passed else 'FAIL'} max_abs={self.max_abs_error:.3g} "
                f"max_rel={self.max_relative_error:.3g} "
                f"failed={self.failed_elements}/{self.total_elements} worst={self.worst_index}")


def compare_outputs(reference: torch.Tensor, candidate: torch.Tensor,
                    rtol: float = 2e-2, atol: float = 2e-3) -> AccuracyReport:
    """Per-element predicate of Ref:289-356: finite AND (|d| <= atol OR
    |d| <= rtol*|ref|).  Deliberately not ``torch.isclose`` (whose
    ``atol + rtol*|ref|`` is looser, Ref:311-313).  Defaults are the
    reference CLI's (Ref:618-619)."""
    if reference.shape != candidate.shape:
        raise AssertionError(f"shape mismatch {tuple(reference.shape)} vs {tuple(candidate.shape)}")
    ref = reference.detach().float()
    opt = candidate.detach().float().to(ref.device)
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    err = (opt - ref).abs()
    ok = finite & ((err <= atol) | (err <= rtol * ref.abs()))
    failed = int((~ok).sum().item())
    err_nan0 = torch.nan_to_num(err, nan=float("inf"))
    flat = int(err_nan0.reshape(-1).argmax().item()) if err.numel() else 0
    idx: List[int] = []
    for size in reversed(ref.shape):
        idx.append(flat % size)
        flat //= size
    rel = err / ref.abs().clamp_min(1e-12)
    return AccuracyReport(
        passed=failed == 0, total_elements=ref.numel(), failed_elements=failed,
        max_abs_error=float(err_nan0.max().item()) if err.numel() else 0.0,
        max_relative_error=float(torch.nan_to_num(rel, nan=float("inf")).max().item()) if err.numel() else 0.0,
        mean_abs_error=float(err.mean().item()) if err.numel() else 0.0,
        worst_index=tuple(reversed(idx)))
