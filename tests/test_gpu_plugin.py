"""The whole reference model with the sm_100a attention sublayer (the
UserOptimizedTransformer drop-in) against the reference's own fp32 output."""

import types

import pytest
import torch

from oracle import compare_outputs
from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef
from tiktok_techjam_2026_track3_b200 import plugin

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_user_optimized_transformer_matches_reference(golden_dir, dtype):
    fx = torch.load(golden_dir / "block_model.pt", weights_only=False)
    cfg = TransformerConfigRef(**fx["config"])
    otb = types.SimpleNamespace(BaselineTransformer=BaselineTransformerRef)
    model = plugin.build(otb, cfg)
    model.load_state_dict(fx["state_dict"], strict=True)
    model = model.to(device="cuda", dtype=dtype).eval()
    x, mask = fx["x"].to(dtype).cuda(), fx["mask"].cuda()
    with torch.inference_mode():
        out = model(x, mask)
    assert out.shape == x.shape
    if dtype == torch.float32:
        # fp32 model: the reference's own output is the target
        rep = compare_outputs(fx["out"], out.float().cpu())
        assert rep.passed, str(rep)
        return
    # 16-bit model: target = the fp32 model on the same rounded weights/inputs.
    ref = BaselineTransformerRef(cfg)
    ref.load_state_dict({k: v.to(dtype).float() for k, v in fx["state_dict"].items()})
    with torch.inference_mode():
        target = ref(fx["x"].to(dtype).float(), fx["mask"])
    if dtype == torch.float16:
        rep = compare_outputs(target, out.float().cpu())
        assert rep.passed, str(rep)
        return
    # bf16: LayerNorm, the FFN and the residual stream run as torch bf16 ops in
    # both models, so the bar is the reference's own bf16 run of the same model
    # (the benchmark's baseline side): our error against fp32 may not exceed it
    # by more than a small factor.
    ref16 = BaselineTransformerRef(cfg)
    ref16.load_state_dict(fx["state_dict"])
    ref16 = ref16.to(device="cuda", dtype=dtype).eval()
    with torch.inference_mode():
        base = ref16(x, mask, in_dtype=True).float().cpu()
    err_ours = (out.float().cpu() - target).abs()
    err_base = (base - target).abs()
    print(f"bf16 model: ours max {err_ours.max():.3g} mean {err_ours.mean():.3g}; "
          f"reference bf16 run max {err_base.max():.3g} mean {err_base.mean():.3g}")
    assert float(err_ours.mean()) <= 1.5 * float(err_base.mean()) + 1e-4
    assert float(err_ours.max()) <= 2.0 * float(err_base.max()) + 1e-3
