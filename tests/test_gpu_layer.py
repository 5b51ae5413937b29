"""The whole attention layer (x + attention(x)) through the C ABI and the
drop-in module, against the fp32 oracle on the same rounded inputs.

Seeds follow the reference benchmark's policy: seeds 1234.. consecutive
(torch_transformer_benchmark.py:382-388), seven of them for benchmark configuration 2.
"""

import pytest
import torch

from oracle import LayerWeights, attention_layer_ref, compare_outputs, generate_case, make_weights
from tiktok_techjam_2026_track3_b200 import B200AttentionLayer, B200SelfAttention, ops

pytestmark = pytest.mark.gpu

DT = {"fp16": torch.float16, "bf16": torch.bfloat16}
FIXTURES = ["cfg1_noncausal", "cfg1_causal", "padded_causal", "ragged_hd128", "tiny_s1"]


def _module(cls, w: LayerWeights, D, H, dtype):
    m = cls(D, H)
    m.load_state_dict({k: v.clone() for k, v in w.state_dict().items()}, strict=True)
    return m.to(device="cuda", dtype=dtype).eval()


def _rounded(w: LayerWeights, dtype):
    return w.to(dtype=dtype).to(dtype=torch.float32)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("name", FIXTURES)
def test_layer_on_golden_inputs(golden_dir, dt, name):
    fx = torch.load(golden_dir / f"attn_{name}.pt", weights_only=False)
    w = LayerWeights.from_state_dict(fx["state_dict"])
    dtype = DT[dt]
    x = fx["x"].to(dtype)
    mask = fx["mask"] if fx["use_mask"] else None
    layer = _module(B200AttentionLayer, w, fx["d_model"], fx["heads"], dtype)
    with torch.inference_mode():
        out = layer(x.cuda(), None if mask is None else mask.cuda(), fx["causal"])
    ref = attention_layer_ref(x.float(), _rounded(w, dtype), fx["heads"], mask, fx["causal"])
    rep = compare_outputs(ref, out.float().cpu())
    assert rep.passed, str(rep)
    # and against the reference's own fp32 output (input rounding included)
    rep32 = compare_outputs(fx["out"], out.float().cpu())
    assert rep32.passed, str(rep32)


@pytest.mark.parametrize("seed", range(1234, 1241))
def test_config2_seven_seeds(seed):
    """benchmark configuration 2 at full size: B8 S2048 D1024 H16 causal fp16."""
    B, S, D, H = 8, 2048, 1024, 16
    x, _ = generate_case(B, S, D, seed, dtype=torch.float16)
    w = make_weights(D, seed, dtype=torch.float16)
    layer = _module(B200AttentionLayer, w.to(dtype=torch.float32), D, H, torch.float16)
    with torch.inference_mode():
        out = layer(x.cuda(), None, True)
        ref = attention_layer_ref(x.cuda(), w.to(dtype=torch.float32, device="cuda"), H, None, True,
                                  batch_chunk=2)
    rep = compare_outputs(ref, out.float())
    assert rep.passed, str(rep)
    ops.check_device_status(out.device)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_padded_masks_and_self_attention_module(dt):
    B, S, D, H = 4, 640, 512, 8
    dtype = DT[dt]
    x, mask = generate_case(B, S, D, 99, dtype=dtype, padding_ratio=0.35)
    w = make_weights(D, 99)
    attn = _module(B200SelfAttention, w, D, H, dtype)
    with torch.inference_mode():
        got = attn(x.cuda(), mask.cuda(), True)
    ref = attention_layer_ref(x.float(), _rounded(w, dtype), H, mask, True, residual=False)
    rep = compare_outputs(ref, got.float().cpu())
    assert rep.passed, str(rep)
    assert torch.count_nonzero(got[~mask.cuda()]) == 0  # masked output rows (Ref :120-121)


def test_forward_residual_matches_block_pattern():
    """residual + attention(norm(x)) as the transformer block computes it."""
    B, S, D, H = 2, 256, 256, 4
    x, _ = generate_case(B, S, D, 5, dtype=torch.float16)
    w = make_weights(D, 5)
    attn = _module(B200SelfAttention, w, D, H, torch.float16)
    xn = torch.nn.functional.layer_norm(x.float(), (D,)).half()
    with torch.inference_mode():
        got = attn.forward_residual(xn.cuda(), x.cuda(), None, True)
    ref = x.float() + attention_layer_ref(xn.float(), _rounded(w, torch.float16), H, None, True,
                                          residual=False)
    assert compare_outputs(ref, got.float().cpu()).passed


def test_weight_cache_invalidation_and_no_aliasing():
    """Anti-cache and aliasing checks of the reference harness: new weights
    take effect, fresh inputs in the same buffer give fresh results, outputs
    are never an internal buffer, inputs are never written."""
    B, S, D, H = 2, 256, 256, 4
    w1, w2 = make_weights(D, 1), make_weights(D, 2)
    layer = _module(B200AttentionLayer, w1, D, H, torch.float16)
    x = generate_case(B, S, D, 3, dtype=torch.float16)[0].cuda()
    x_copy = x.clone()
    with torch.inference_mode():
        o1 = layer(x, None, True)
        o1b = layer(x, None, True)
    assert o1.data_ptr() != o1b.data_ptr() and torch.equal(o1, o1b)
    assert torch.equal(x, x_copy)
    layer.load_state_dict({k: v.half().cuda() for k, v in w2.state_dict().items()})
    with torch.inference_mode():
        o2 = layer(x, None, True)
        x.copy_(generate_case(B, S, D, 4, dtype=torch.float16)[0].cuda())
        o3 = layer(x, None, True)
    ref2 = attention_layer_ref(x_copy.float(), _rounded(w2, torch.float16), H, None, True)
    ref3 = attention_layer_ref(x.float(), _rounded(w2, torch.float16), H, None, True)
    assert compare_outputs(ref2, o2.float()).passed
    assert compare_outputs(ref3, o3.float()).passed
    assert not torch.equal(o1, o2)


def test_unsupported_inputs_raise():
    layer = B200AttentionLayer(256, 4).cuda().half()
    with pytest.raises(RuntimeError, match="dtype"):
        layer(torch.randn(1, 8, 256, device="cuda"), None, True)   # fp32 input
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        B200AttentionLayer(256, 4).half()(torch.randn(1, 8, 256).half(), None, True)
    with pytest.raises(RuntimeError, match="head_dim"):   # head_dim 12: not a multiple of 8
        B200AttentionLayer(96, 8).cuda().half()(torch.randn(1, 8, 96, device="cuda").half())
    with pytest.raises(RuntimeError, match="head_dim"):   # head_dim 512 > 256
        B200AttentionLayer(512, 1).cuda().half()(torch.randn(1, 8, 512, device="cuda").half())
