"""B200-native (sm_100a) attention-layer forward, a drop-in for the attention
path of yyan115/Tiktok_TechJam_2026_Track3's ``torch_transformer_benchmark.py``.

Host side: Python/PyTorch modules with the reference's parameter names and
forward signature.  Device side: ``libttj_attn_sm100.so`` (C ABI in
``include/ttj_attn.h``) with tcgen05/TMEM GEMMs fed by TMA and a flash-attention
kernel.  No CPU fallback: without the built library every op raises.
"""

from . import ops  # noqa: F401
from .config import PRESETS, LayerConfig, attention_flops  # noqa: F401
from .layer import B200AttentionLayer, B200SelfAttention  # noqa: F401

__version__ = "0.1.0"
