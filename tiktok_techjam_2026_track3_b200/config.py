"""Shape records for the attention layer and the five benchmark workloads.

``LayerConfig`` mirrors the fields of the reference's ``TransformerConfig``
(torch_transformer_benchmark.py:29-56) that the attention layer uses, plus the
dtype / quantisation / sharding choices of each workload, and validates the
same way (positive sizes, ``d_model % num_heads == 0``) before adding the
kernels' own limits.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Dict, Optional

import torch

__all__ = ["LayerConfig", "PRESETS", "DTYPES", "attention_flops", "ModelShape", "OFFICIAL_SHAPES"]

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


@dataclass(frozen=True)
class LayerConfig:
    name: str
    batch: int
    seq_len: int
    d_model: int
    num_heads: int
    causal: bool
    dtype: str = "float16"
    quant: Optional[str] = None      # None or "int8" (W8A8 projections)
    shard: str = "batch"             # how bench / partitioner split it over GPUs
    scaling: str = "weak"            # multi-GPU bench: "weak" (batch per GPU) or "strong" (batch split)
    input_scale: float = 1.0
    weight_std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    @property
    def tokens(self) -> int:
        return self.batch * self.seq_len

    @property
    def torch_dtype(self) -> torch.dtype:
        return DTYPES[self.dtype]

    def validate(self) -> None:
        if min(self.batch, self.seq_len, self.d_model, self.num_heads) <= 0:
            raise ValueError("batch, seq_len, d_model and num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(f"d_model ({self.d_model}) must be divisible by num_heads ({self.num_heads})")
        if self.head_dim % 8 != 0 or self.head_dim > 256:
            raise ValueError("head_dim must be a multiple of 8 and at most 256 for the sm_100a kernels")
        if self.d_model % 32 != 0:
            raise ValueError("d_model must be a multiple of 32")
        if self.dtype not in DTYPES:
            raise ValueError(f"dtype must be one of {sorted(DTYPES)}")
        if self.quant not in (None, "int8"):
            raise ValueError("quant must be None or 'int8'")
        if self.shard not in ("batch", "heads"):
            raise ValueError("shard must be 'batch' or 'heads'")
        if self.scaling not in ("weak", "strong"):
            raise ValueError("scaling must be 'weak' or 'strong'")

    def with_(self, **kw) -> "LayerConfig":
        return replace(self, **kw)


def attention_flops(cfg: LayerConfig, include_projections: bool = True) -> float:
    """Algorithmic FLOPs of one layer forward: 2*T*D*3D (QKV) + 2*T*D*D (out)
    + 4*B*H*S^2*hd, halved for causal (the counting rule of the reference's
    Project/loop/ceiling.py:44-45, :93-97, without the FFN)."""
    T, D = cfg.tokens, cfg.d_model
    attn = 4.0 * cfg.batch * cfg.num_heads * cfg.seq_len ** 2 * cfg.head_dim
    if cfg.causal:
        attn *= 0.5
    proj = 2.0 * T * D * 3 * D + 2.0 * T * D * D if include_projections else 0.0
    return attn + proj


PRESETS: Dict[int, LayerConfig] = {
    1: LayerConfig("cfg1_cpu_fp32_b2_s128_d256_h4", 2, 128, 256, 4, causal=False,
                   dtype="float32", input_scale=0.02),
    2: LayerConfig("cfg2_fp16_b8_s2048_d1024_h16_causal", 8, 2048, 1024, 16, causal=True,
                   dtype="float16"),
    3: LayerConfig("cfg3_int8_b16_s4096_d4096_h32_causal", 16, 4096, 4096, 32, causal=True,
                   dtype="bfloat16", quant="int8", scaling="strong"),
    4: LayerConfig("cfg4_bf16_b32_s100000_d512_h8_causal", 32, 100000, 512, 8, causal=True,
                   dtype="bfloat16", scaling="strong"),
    5: LayerConfig("cfg5_bf16_b1_s262144_d4096_h32_causal", 1, 262144, 4096, 32, causal=True,
                   dtype="bfloat16", shard="heads", scaling="strong"),
}


@dataclass(frozen=True)
class ModelShape:
    """One whole-model benchmark shape: the CLI dials of the reference's
    torch_transformer_benchmark.py (--batch-size, --d-model, --heads, --seq-len,
    --layers, --ffn-dim; every official shape passes --causal)."""
    batch: int
    d_model: int
    num_heads: int
    seq_len: int
    num_layers: int
    ffn_dim: int
    causal: bool = True

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads


# The 14 official test shapes of the reference (Project/shapes.json, ids 1-14).
# head_dim spans 8 (ids 7, 11), 32 (ids 1-6, 12, 13), 64 (ids 10, 14),
# 128 (id 9) and 256 (id 8).  Id 14 cannot run through the dense reference.
OFFICIAL_SHAPES: Dict[int, ModelShape] = {
    1: ModelShape(64, 128, 4, 128, 4, 128),
    2: ModelShape(1, 128, 4, 128, 4, 128),
    3: ModelShape(4, 128, 4, 128, 4, 128),
    4: ModelShape(16, 128, 4, 128, 4, 128),
    5: ModelShape(128, 128, 4, 128, 4, 128),
    6: ModelShape(10000, 128, 4, 128, 4, 128),
    7: ModelShape(64, 32, 4, 128, 4, 32),
    8: ModelShape(64, 1024, 4, 128, 4, 1024),
    9: ModelShape(64, 128, 1, 128, 4, 128),
    10: ModelShape(64, 128, 2, 128, 4, 128),
    11: ModelShape(64, 128, 16, 128, 4, 128),
    12: ModelShape(64, 128, 4, 32, 4, 128),
    13: ModelShape(64, 128, 4, 1024, 4, 128),
    14: ModelShape(32, 1024, 16, 100000, 2, 1024),
}
