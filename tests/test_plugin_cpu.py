"""The harness-facing drop-in without a GPU: module tree and state-dict keys
equal the reference model's, strict load_state_dict works."""

import types

import torch

from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef
from tiktok_techjam_2026_track3_b200 import plugin


def test_build_keeps_reference_state_dict(golden_dir):
    fx = torch.load(golden_dir / "block_model.pt", weights_only=False)
    cfg = TransformerConfigRef(**fx["config"])
    otb = types.SimpleNamespace(BaselineTransformer=BaselineTransformerRef)
    model = plugin.build(otb, cfg)
    assert type(model).__name__ == "UserOptimizedTransformer"
    assert isinstance(model, BaselineTransformerRef)
    ref = BaselineTransformerRef(cfg)
    assert list(model.state_dict().keys()) == list(ref.state_dict().keys())
    model.load_state_dict(fx["state_dict"], strict=True)
    # the attention view shares the block's Linear modules and adds no keys
    attn = plugin.attention_sublayer(model.layers[0])
    assert attn.q_proj is model.layers[0].attention.q_proj
    assert list(model.state_dict().keys()) == list(ref.state_dict().keys())


def test_official_shapes_table_matches_reference_manifest():
    """config.OFFICIAL_SHAPES restates the reference's Project/shapes.json (read
    here only when the reference checkout is present; it never travels)."""
    import json
    from pathlib import Path

    import pytest

    from tiktok_techjam_2026_track3_b200.config import OFFICIAL_SHAPES
    manifest = Path("/root/reference/Project/shapes.json")
    if not manifest.exists():
        pytest.skip("reference checkout not present")
    shapes = json.loads(manifest.read_text())["shapes"]
    assert sorted(OFFICIAL_SHAPES) == sorted(s["id"] for s in shapes)
    for s in shapes:
        m = OFFICIAL_SHAPES[s["id"]]
        assert (m.batch, m.d_model, m.num_heads, m.seq_len, m.num_layers, m.ffn_dim, m.causal) == (
            s["batch_size"], s["d_model"], s["num_heads"], s["seq_len"], s["num_layers"], s["ffn_dim"],
            s["causal"])


def test_block_parameter_dtypes_for_each_model_dtype():
    """16-bit models keep every block parameter in their dtype; fp32 models keep the
    LayerNorm parameters and the residual-side biases in fp32 (the fp32 residual
    stream) and the tensor-core operands in fp16."""
    from tiktok_techjam_2026_track3_b200 import ops
    for dt in (torch.float16, torch.bfloat16):
        assert all(ops.block_param_dtype(n, dt) == dt for n in ops.BLOCK_PARAMS)
    f32 = {n for n in ops.BLOCK_PARAMS if ops.block_param_dtype(n, torch.float32) == torch.float32}
    assert f32 == {"ln1_w", "ln1_b", "b_o", "ln2_w", "ln2_b", "b_out"}
    assert all(ops.block_param_dtype(n, torch.float32) == torch.float16 for n in ops.BLOCK_PARAMS if n not in f32)
