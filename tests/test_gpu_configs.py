"""Every benchmark configuration at its own size on seeds 1234-1240 (the
reference benchmark's consecutive-seed policy, torch_transformer_benchmark.py:382-388),
through the drop-in layer module, against the oracle.  Configuration 2 is in
test_gpu_layer.py.

What is compared, per dtype:

* fp16 and the fp32 configuration: the reference predicate (abs 2e-3 OR rel 2e-2
  per element, Ref :306-318) against the fp32 layer on the inputs the kernels see.
* bf16: bf16 keeps 8 significant bits.  At d_model 4096 the reference's own bf16
  run cannot meet 2e-3 against fp32: rounding the context to bf16 before the
  4096-term out-projection alone moves outputs by ~2.6e-3 (RMS) in rows that
  attend to few keys, so ~2% of elements fail the predicate (5.8% of the first
  64 rows of a sequence).  The gate there is "no worse than the reference's own
  bf16 rounding": the oracle evaluated with bf16 storage wherever the reference's
  bf16 run stores a tensor (``attention_layer_rows_ref``) is compared against fp32
  too, and the kernels may not fail more elements, nor have a larger mean or
  maximum error, than it does (within a small margin).  Where that bf16-storage
  oracle passes the predicate outright (d_model 512), the gate is the predicate
  itself.  Both reports are printed.
* int8 (configuration 3): the integer stages bit for bit, the attention stage
  with the bf16 rule above, the end-to-end distance to the recipe reported.
"""

import pytest
import torch

from oracle import (attention_layer_ref, attention_layer_rows_ref, compare_outputs, generate_case,
                    int8_attention_layer_ref, int8_linear_ref, make_weights, quant_rows_ref,
                    quant_weight_ref)
from parity_util import no_worse_than_reference_rounding
from tiktok_techjam_2026_track3_b200 import B200AttentionLayer, ops
from tiktok_techjam_2026_track3_b200.config import PRESETS

pytestmark = pytest.mark.gpu

SEEDS = list(range(1234, 1241))


def _layer(cfg, w, quant=None):
    m = B200AttentionLayer(cfg.d_model, cfg.num_heads, quant=quant)
    m.load_state_dict(w.state_dict(), strict=True)
    return m.to(device="cuda", dtype=cfg.torch_dtype).eval()


# ------------------------------------------------------------------ config 1
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("seed", SEEDS)
def test_config1_fp32_layer(seed, dt):
    """B2 S128 D256 H4 non-causal, inputs and weights N(0,1)*0.02 (the fp32 CPU
    configuration): the layer in 16-bit against the reference's fp32 output on
    the unrounded inputs."""
    cfg = PRESETS[1]
    x, _ = generate_case(cfg.batch, cfg.seq_len, cfg.d_model, seed, input_scale=cfg.input_scale)
    w = make_weights(cfg.d_model, seed)
    layer = _layer(cfg.with_(dtype={torch.float16: "float16", torch.bfloat16: "bfloat16"}[dt]), w)
    with torch.inference_mode():
        out = layer(x.to(dt).cuda(), None, cfg.causal)
    ref = attention_layer_ref(x, w, cfg.num_heads, None, cfg.causal)
    rep = compare_outputs(ref, out.float().cpu())
    assert rep.passed, str(rep)


# ------------------------------------------------------------------ configs 4 and 5
def _stripes(S, seed):
    g = torch.Generator().manual_seed(seed)
    mid = int(torch.randint(64, S - 128, (1,), generator=g))
    return torch.cat([torch.arange(0, 64), torch.arange(mid, mid + 64), torch.arange(S - 64, S)])


@pytest.mark.parametrize("cid", [4, 5])
@pytest.mark.parametrize("seed", SEEDS)
def test_long_context_layer_stripes(cid, seed):
    """Configuration 4 (B32 S100000 D512 H8 hd64) and 5 (B1 S262144 D4096 H32
    hd128), bf16, causal, at full size: the whole layer (QKV projection,
    attention, out-projection with bias and residual) runs on the GPU; the
    oracle evaluates the first 64 rows, 64 rows at a seeded offset and the last
    64 rows of two batch rows (all heads), streaming over every key they see."""
    cfg = PRESETS[cid]
    B, S, D, H = cfg.batch, cfg.seq_len, cfg.d_model, cfg.num_heads
    x, _ = generate_case(B, S, D, seed, dtype=cfg.torch_dtype, device="cuda")
    w = make_weights(D, seed)
    layer = _layer(cfg, w)
    with torch.inference_mode():
        out = layer(x, None, cfg.causal)
    torch.cuda.synchronize()
    ops.check_device_status(out.device)
    batches = sorted({seed % B, (seed * 7 + 3) % B})
    rows = _stripes(S, seed)
    wr = w.to(dtype=cfg.torch_dtype).to(dtype=torch.float32, device="cuda")
    with torch.inference_mode():
        ref32, ref16 = attention_layer_rows_ref(x, wr, H, cfg.causal, batches, rows,
                                                store_dtypes=(None, cfg.torch_dtype))
    got = out[batches][:, rows.cuda()].float()
    no_worse_than_reference_rounding(ref32, got, ref16, f"cfg{cid} seed {seed}")
    if cid == 4:  # the bf16-storage oracle meets the predicate at d_model 512: so must the kernels
        assert compare_outputs(ref32, got).passed


@pytest.mark.parametrize("seed", [1234, 1235])
def test_config5_shape_in_fp16_meets_the_predicate(seed):
    """The same d_model-4096 long-context layer in fp16 (11 significant bits):
    here the predicate against fp32 is attainable and must hold."""
    cfg = PRESETS[5].with_(dtype="float16")
    B, S, D, H = cfg.batch, cfg.seq_len, cfg.d_model, cfg.num_heads
    x, _ = generate_case(B, S, D, seed, dtype=torch.float16, device="cuda")
    w = make_weights(D, seed)
    layer = _layer(cfg, w)
    with torch.inference_mode():
        out = layer(x, None, True)
    rows = _stripes(S, seed)
    wr = w.to(dtype=torch.float16).to(dtype=torch.float32, device="cuda")
    with torch.inference_mode():
        (ref32,) = attention_layer_rows_ref(x, wr, H, True, [0], rows)
    rep = compare_outputs(ref32, out[[0]][:, rows.cuda()].float())
    assert rep.passed, str(rep)


# ------------------------------------------------------------------ config 3 (int8)
def _attention_dense(qkv, H, causal, probs_dtype=None):
    """fp32 attention of one batch row's packed qkv [S, 3D], head by head;
    probs_dtype rounds the normalised probabilities as the reference's 16-bit
    run does (torch_transformer_benchmark.py:111)."""
    S, D3 = qkv.shape
    D = D3 // 3
    hd = D // H
    out = torch.empty(S, D, device=qkv.device)
    causal_mask = torch.ones(S, S, dtype=torch.bool, device=qkv.device).triu(1)
    for h in range(H):
        q, k, v = (qkv[:, o * D + h * hd:o * D + (h + 1) * hd].float() for o in range(3))
        s = q @ k.T * hd ** -0.5
        if causal:
            s = s.masked_fill(causal_mask, float("-inf"))
        p = torch.softmax(s, -1)
        if probs_dtype is not None:
            p = p.to(probs_dtype).float()
        out[:, h * hd:(h + 1) * hd] = p @ v
    return out


@pytest.mark.parametrize("seed", SEEDS)
def test_config3_int8_layer(seed):
    """B16 S4096 D4096 H32 causal, W8A8 projections with bf16 attention, full
    batch on the GPU.  One batch row per seed (a different one each seed) is
    checked stage by stage: the per-token quantiser, the int32 GEMM and the
    dequant epilogue bit for bit against the recipe (k008_int8_gemm.py:148-185),
    the attention stage against fp32 with the bf16 rule, the out-projection and
    residual bit for bit given the kernel's context."""
    cfg = PRESETS[3]
    B, S, D, H = cfg.batch, cfg.seq_len, cfg.d_model, cfg.num_heads
    T = B * S
    x, _ = generate_case(B, S, D, seed, dtype=torch.bfloat16, device="cuda")
    w = make_weights(D, seed)
    layer = _layer(cfg, w, quant="int8")
    w8, s8, b32, wo8, so8, bo32 = layer.packed_weights()
    with torch.inference_mode():
        out = layer(x, None, True)
        a8, s_a = ops.int8_quant_rows(x.view(T, D))
        qkv = ops.int8_linear(a8, s_a, w8, s8, b32, torch.bfloat16).view(B, S, 3 * D)
        ctx = ops.flash_attn(qkv, H, True)
        c8, s_c = ops.int8_quant_rows(ctx.view(T, D))
        staged = ops.int8_linear(c8, s_c, wo8, so8, bo32, torch.bfloat16, residual=x.view(T, D)).view(B, S, D)
    ops.check_device_status(x.device)
    assert torch.equal(out, staged)  # the layer call is exactly the staged composition
    b = (seed - 1234) * 2 + 1
    wb = w.to(dtype=torch.bfloat16).to(dtype=torch.float32, device="cuda")
    wqkv = torch.cat([wb.wq, wb.wk, wb.wv], 0)
    bqkv = torch.cat([wb.bq, wb.bk, wb.bv], 0)
    wq8_ref, sq_ref = quant_weight_ref(wqkv)
    assert torch.equal(w8, wq8_ref) and torch.equal(s8, sq_ref)
    xb = x[b].float()
    a8_ref, sa_ref = quant_rows_ref(xb)
    assert torch.equal(a8.view(B, S, D)[b], a8_ref) and torch.equal(s_a.view(B, S)[b], sa_ref)
    qkv_ref = int8_linear_ref(xb, wq8_ref, sq_ref, bqkv).to(torch.bfloat16)
    assert torch.equal(qkv[b], qkv_ref)
    # attention stage on the kernel's own qkv of this row
    ref32 = _attention_dense(qkv[b], H, True)
    ref16 = _attention_dense(qkv[b], H, True, probs_dtype=torch.bfloat16).to(torch.bfloat16).float()
    no_worse_than_reference_rounding(ref32, ctx[b].float(), ref16, f"cfg3 attention seed {seed}")
    # out-projection + residual given the kernel's context: bit-exact
    wo8_ref, so_ref = quant_weight_ref(wb.wo)
    out_ref = xb + int8_linear_ref(ctx[b].float(), wo8_ref, so_ref, wb.bo)
    assert torch.equal(out[b], out_ref.to(torch.bfloat16))
    # end to end against the recipe evaluated with fp32 attention (reported, loosely bounded:
    # per-token requantisation of the context turns sub-step differences into flipped roundings)
    e2e = compare_outputs(int8_attention_layer_ref(x[b:b + 1], wb, H, True), out[b:b + 1].float())
    print(f"cfg3 seed {seed} row {b}: end to end vs the recipe with fp32 attention: {e2e}")
    assert e2e.max_abs_error < 0.1 and e2e.mean_abs_error < 5e-3
