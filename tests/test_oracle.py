"""The oracle against the golden vectors written from the reference's own code.

CPU only.  tests/golden/*.pt were produced by tests/golden/make_golden.py,
which imports the reference's torch_transformer_benchmark.py and
Project/kernels/k008_int8_gemm.py unmodified.
"""

import pytest
import torch

from oracle import (LayerWeights, attention_layer_ref, attention_layer_rows_ref,
                    attention_layer_streamed_ref, compare_outputs, generate_case, int8_linear_ref,
                    int_gemm_ref, make_weights, quant_rows_ref, quant_weight_ref, split_heads,
                    streamed_attention_ref)

ATTN_FIXTURES = ["cfg1_noncausal", "cfg1_causal", "padded_causal", "ragged_hd128", "tiny_s1"]


def load(golden_dir, name):
    return torch.load(golden_dir / f"{name}.pt", weights_only=False)


@pytest.mark.parametrize("name", ATTN_FIXTURES)
def test_generator_matches_reference(golden_dir, name):
    fx = load(golden_dir, f"attn_{name}")
    x, mask = generate_case(fx["batch"], fx["seq_len"], fx["d_model"], fx["seed"],
                            padding_ratio=fx["padding_ratio"])
    assert torch.equal(x, fx["x"])
    assert torch.equal(mask, fx["mask"])


@pytest.mark.parametrize("name", ATTN_FIXTURES)
def test_dense_oracle_matches_reference(golden_dir, name):
    fx = load(golden_dir, f"attn_{name}")
    w = LayerWeights.from_state_dict(fx["state_dict"])
    mask = fx["mask"] if fx["use_mask"] else None
    out = attention_layer_ref(fx["x"], w, fx["heads"], mask, fx["causal"])
    torch.testing.assert_close(out, fx["out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ATTN_FIXTURES)
def test_streamed_oracle_matches_reference(golden_dir, name):
    """Streamed (online-softmax) attention equals the reference on every row."""
    fx = load(golden_dir, f"attn_{name}")
    w = LayerWeights.from_state_dict(fx["state_dict"])
    x = fx["x"]
    B, S, D = x.shape
    H = fx["heads"]
    mask = fx["mask"] if fx["use_mask"] else None
    q = split_heads(torch.nn.functional.linear(x, w.wq, w.bq), H)
    k = split_heads(torch.nn.functional.linear(x, w.wk, w.bk), H)
    v = split_heads(torch.nn.functional.linear(x, w.wv, w.bv), H)
    ctx = torch.empty_like(q)
    for b in range(B):
        for h in range(H):
            ctx[b, h] = streamed_attention_ref(q[b, h], k[b, h], v[b, h], (D // H) ** -0.5,
                                               fx["causal"], None if mask is None else mask[b],
                                               k_chunk=32)
    out = torch.nn.functional.linear(ctx.transpose(1, 2).reshape(B, S, D), w.wo, w.bo)
    if mask is not None:
        out = out.masked_fill(~mask[..., None], 0)
    torch.testing.assert_close(x + out, fx["out"], rtol=1e-5, atol=1e-5)


def test_streamed_matches_dense_long():
    """The long-context checker against dense attention at S up to 1024 (the
    validation gate the reference applies to its own streamed oracle)."""
    g = torch.Generator().manual_seed(7)
    for S, causal in ((1024, True), (700, False)):
        q, k, v = (torch.randn(S, 64, generator=g) for _ in range(3))
        dense = torch.softmax(
            (q @ k.T * 0.125).masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
            if causal else q @ k.T * 0.125, -1) @ v
        rows = torch.tensor([0, 1, 127, 128, S // 2, S - 1])
        got = streamed_attention_ref(q[rows], k, v, 0.125, causal, q_rows=rows, k_chunk=256)
        torch.testing.assert_close(got, dense[rows], rtol=1e-5, atol=1e-5)


def test_sampled_stripe_oracle_matches_dense(golden_dir):
    fx = load(golden_dir, "attn_cfg1_causal")
    w = LayerWeights.from_state_dict(fx["state_dict"])
    x = fx["x"]
    H = fx["heads"]
    rows = torch.tensor([0, 5, 64, 127])
    got = attention_layer_streamed_ref(x, w, H, True, [1], [2], rows, k_chunk=48)
    q = split_heads(torch.nn.functional.linear(x, w.wq, w.bq), H)
    k = split_heads(torch.nn.functional.linear(x, w.wk, w.bk), H)
    v = split_heads(torch.nn.functional.linear(x, w.wv, w.bv), H)
    s = (q @ k.transpose(-1, -2)) * (x.shape[-1] // H) ** -0.5
    s = s.masked_fill(torch.ones(128, 128, dtype=torch.bool).triu(1), float("-inf"))
    dense = torch.softmax(s, -1) @ v
    torch.testing.assert_close(got[0, 0], dense[1, 2, rows], rtol=1e-5, atol=1e-6)


def test_predicate_semantics():
    ref = torch.tensor([1.0, 0.0, 100.0, float("nan")])
    assert compare_outputs(ref[:3], ref[:3]).passed
    # abs-only passes near zero, rel-only passes for large values, OR not sum
    assert compare_outputs(torch.tensor([0.0]), torch.tensor([0.0019])).passed
    assert not compare_outputs(torch.tensor([0.0]), torch.tensor([0.0021])).passed
    assert compare_outputs(torch.tensor([100.0]), torch.tensor([101.9])).passed
    assert not compare_outputs(torch.tensor([100.0]), torch.tensor([102.1])).passed
    # isclose would accept atol + rtol*|ref| = 0.002 + 0.02; the OR rule does not
    assert not compare_outputs(torch.tensor([1.0]), torch.tensor([1.021])).passed
    assert not compare_outputs(ref, ref).passed  # non-finite fails


def test_planted_mistake_is_caught(golden_dir):
    """A wrong result (planted in the oracle's output, on the CPU) must fail."""
    fx = load(golden_dir, "attn_cfg1_noncausal")
    w = LayerWeights.from_state_dict(fx["state_dict"])
    out = attention_layer_ref(fx["x"], w, fx["heads"], None, False)
    bad = out.clone()
    bad[1, 17, 3] += 0.05
    rep = compare_outputs(fx["out"], bad)
    assert not rep.passed and rep.failed_elements == 1 and rep.worst_index == (1, 17, 3)
    # causal vs non-causal confusion is caught too
    wrong = attention_layer_ref(fx["x"], w, fx["heads"], None, True)
    assert not compare_outputs(fx["out"], wrong).passed


def test_int8_recipe_bit_exact(golden_dir):
    fx = load(golden_dir, "int8_recipe")
    a8, s_a = quant_rows_ref(fx["h"])
    assert torch.equal(a8, fx["a8"])
    assert torch.equal(s_a, fx["s_a"])
    w8, s_w = quant_weight_ref(fx["weight"])
    assert torch.equal(w8, fx["w8"])
    assert torch.equal(s_w, fx["s_w"])
    assert torch.equal(int_gemm_ref(a8, w8), fx["acc"])
    y = int8_linear_ref(fx["h"], w8, s_w, fx["bias"])
    assert torch.equal(y, fx["y"])


def test_block_oracle_matches_reference_model(golden_dir):
    """The whole-model restatement (blocks + final norm) against the reference's
    BaselineTransformer output."""
    from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef
    fx = torch.load(golden_dir / "block_model.pt", weights_only=False)
    model = BaselineTransformerRef(TransformerConfigRef(**fx["config"]))
    model.load_state_dict(fx["state_dict"], strict=True)
    with torch.inference_mode():
        out = model(fx["x"], fx["mask"])
    torch.testing.assert_close(out, fx["out"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("seq,batch", [(1024, 2), (2048, 2), (4096, 1)])
def test_streamed_checker_gate_whole_model(seq, batch):
    """The reference's own gate for its long-context checker
    (Project/tools/shape14_eval.py:279-316): the whole model of official shape
    14 (d_model 1024, 16 heads, ffn 1024, 2 layers, causal) evaluated by
    ``streamed_model_ref`` against the dense model, S in {1024, 2048, 4096},
    three seeds each, max |diff| < 1e-3 in fp32.  The chunk sizes divide
    neither S nor each other, so ragged query and key chunks are exercised."""
    from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef, streamed_model_ref
    cfg = TransformerConfigRef(batch_size=batch, seq_len=seq, d_model=1024, num_heads=16, ffn_dim=1024,
                               num_layers=2, causal=True)
    torch.manual_seed(seq)
    dense = BaselineTransformerRef(cfg).eval()
    for seed in (1234, 1235, 1236):
        x, mask = generate_case(batch, seq, 1024, seed)
        with torch.inference_mode():
            err = (streamed_model_ref(dense, x, mask, q_chunk=700, k_chunk=1100) - dense(x, mask)).abs().max().item()
        assert err < 1e-3, (seq, seed, err)


@pytest.mark.parametrize("causal", [True, False])
def test_streamed_model_with_padding_and_small_chunks(causal):
    """``streamed_model_ref`` with prefix key masks (padded rows zeroed, the
    reference's generator at padding 0.4) and chunks of a few rows, against the
    dense model to 1e-5."""
    from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef, streamed_model_ref
    cfg = TransformerConfigRef(batch_size=3, seq_len=200, d_model=64, num_heads=4, ffn_dim=96,
                               num_layers=2, causal=causal)
    torch.manual_seed(7)
    dense = BaselineTransformerRef(cfg).eval()
    x, mask = generate_case(3, 200, 64, 1240, padding_ratio=0.4)
    assert not bool(mask.all())
    with torch.inference_mode():
        ref = dense(x, mask)
        got = streamed_model_ref(dense, x, mask, q_chunk=37, k_chunk=23)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
    assert bool((got[~mask] == 0).all())


def test_rows_ref_matches_dense_layer_and_rounding_points():
    """attention_layer_rows_ref against the dense oracle (fp32), and its 16-bit
    variant against a dense restatement that rounds at the same points."""
    B, S, D, H = 2, 300, 256, 4
    x, mask = generate_case(B, S, D, 11, padding_ratio=0.3)
    x = x.to(torch.bfloat16).float()
    w = make_weights(D, 11).to(dtype=torch.bfloat16).to(dtype=torch.float32)
    rows = torch.tensor([0, 1, 2, 77, 150, 255, 299])
    for causal in (True, False):
        got32, got16 = attention_layer_rows_ref(x, w, H, causal, [0, 1], rows,
                                                store_dtypes=(None, torch.bfloat16),
                                                valid_token_mask=mask, k_chunk=64)
        dense = attention_layer_ref(x, w, H, mask, causal)
        torch.testing.assert_close(got32, dense[:, rows], rtol=1e-5, atol=1e-5)

        def r(t):
            return t.to(torch.bfloat16).float()
        q, k, v = (r(split_heads(torch.nn.functional.linear(x, a, b), H))
                   for a, b in ((w.wq, w.bq), (w.wk, w.bk), (w.wv, w.bv)))
        sc = q @ k.transpose(-1, -2) * (D // H) ** -0.5
        if causal:
            sc = sc.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
        sc = sc.masked_fill(~mask[:, None, None, :], float("-inf"))
        ctx = r(r(torch.softmax(sc, -1)) @ v).transpose(1, 2).reshape(B, S, D)
        o = r(torch.nn.functional.linear(ctx, w.wo, w.bo)).masked_fill(~mask[..., None], 0)
        ref16 = r(x + o)
        torch.testing.assert_close(got16, ref16[:, rows], rtol=0, atol=2 ** -7)
        # almost every element is the identical 16-bit value (accumulation order aside)
        assert float((got16 == ref16[:, rows]).float().mean()) > 0.97
