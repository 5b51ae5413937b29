"""The reference's official benchmark shapes (Project/shapes.json) through the
drop-in model, ``plugin.build(otb, config)``, against the whole-model oracle.

Eleven of the fourteen shapes use head_dim 8, 32 or 256 (and shape 7 d_model
32); they run on the padded attention kernels.  Batch rows never interact, so
each shape runs at a reduced batch (the sequence length, widths, head count,
depth and ffn_dim are the shape's own).  fp16 models are checked with the
reference predicate (abs 2e-3 OR rel 2e-2) against the fp32 model on the same
rounded weights and inputs; fp32 models (the benchmark's default dtype, whose
attention sublayer runs with fp16 operands) against the reference's fp32 output.
"""

import types

import pytest
import torch

from oracle import compare_outputs, generate_case
from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef
from tiktok_techjam_2026_track3_b200 import plugin
from tiktok_techjam_2026_track3_b200.config import OFFICIAL_SHAPES

pytestmark = pytest.mark.gpu

OTB = types.SimpleNamespace(BaselineTransformer=BaselineTransformerRef)


def _models(sid, batch):
    sh = OFFICIAL_SHAPES[sid]
    cfg = TransformerConfigRef(batch_size=batch, seq_len=sh.seq_len, d_model=sh.d_model,
                               num_heads=sh.num_heads, ffn_dim=sh.ffn_dim, num_layers=sh.num_layers,
                               causal=sh.causal)
    torch.manual_seed(1000 + sid)
    ref = BaselineTransformerRef(cfg).eval()  # nn.Linear / nn.LayerNorm default init, as the reference
    model = plugin.build(OTB, cfg)
    model.load_state_dict(ref.state_dict(), strict=True)
    return cfg, ref, model


@pytest.mark.parametrize("padding", [0.0, 0.25])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("sid", [1, 2, 7, 8, 9, 10, 11, 12, 13])
def test_official_shape_through_plugin(sid, dtype, padding):
    batch = min(OFFICIAL_SHAPES[sid].batch, 2 if sid == 13 else 4)
    cfg, ref, model = _models(sid, batch)
    x, mask = generate_case(batch, cfg.seq_len, cfg.d_model, 1234 + sid, padding_ratio=padding)
    model = model.to(device="cuda", dtype=dtype).eval()
    with torch.inference_mode():
        out = model(x.to(dtype).cuda(), mask.cuda())
    if dtype == torch.float32:
        with torch.inference_mode():
            target = ref(x, mask)
    else:
        r16 = BaselineTransformerRef(cfg)
        r16.load_state_dict({k: v.to(dtype).float() for k, v in ref.state_dict().items()})
        with torch.inference_mode():
            target = r16(x.to(dtype).float(), mask)
    rep = compare_outputs(target, out.float().cpu())
    assert rep.passed, f"shape {sid} B{batch} {dtype}: {rep}"
    assert bool((out[~mask.cuda()] == 0).all())  # masked rows zeroed (Ref :170-171)
