"""CPU oracle for the attention-layer forward (test infrastructure only).

This package restates, in fp32 PyTorch on the CPU, the algorithm the reference
benchmark times for one transformer attention layer:
``x + out_proj(SDPA(split_heads(x Wq^T + bq), ...)))``.

It is the CHECKER, never the product. Only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product path (``tiktok_techjam_2026_track3_b200``) never imports this package
and fails loudly when its CUDA library is missing.

Parity status: pinned. ``tests/golden/make_golden.py`` imports the reference's own
``torch_transformer_benchmark.py`` (``BaselineSelfAttention``, ``generate_random_case``)
and the reference's int8 recipe (``Project/kernels/k008_int8_gemm.py``) to write the
fixtures under ``tests/golden/``; ``tests/test_oracle.py`` checks this package
against them.
"""

from .attention_ref import (  # noqa: F401
    AccuracyReport,
    LayerWeights,
    attention_layer_ref,
    attention_layer_rows_ref,
    attention_layer_streamed_ref,
    compare_outputs,
    generate_case,
    make_weights,
    streamed_attention_ref,
    split_heads,
)
from .int8_ref import (  # noqa: F401
    int8_attention_layer_ref,
    int8_linear_ref,
    int_gemm_ref,
    quant_rows_ref,
    quant_weight_ref,
)
