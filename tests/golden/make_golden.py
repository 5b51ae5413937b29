"""Write the golden fixtures under tests/golden/ from the REFERENCE's own code.

Usage (needs a checkout of the reference repository; it is not needed to run
the tests, only to regenerate the fixtures):

    python tests/golden/make_golden.py --reference <path to reference checkout>

What it imports from the reference, unmodified:

* ``torch_transformer_benchmark.py``: ``BaselineSelfAttention`` (the layer),
  ``generate_random_case`` (seeded inputs and prefix masks) and
  ``compare_outputs`` is not needed (fixtures store raw tensors);
* ``Project/kernels/k008_int8_gemm.py``: ``_quant_rows``, ``_int8_pack`` and
  ``_int8_linear`` (the W8A8 recipe);
* ``BaselineTransformer`` for one whole-model fixture (``block_model.pt``).

Each attention fixture stores the reference's inputs, the state dict it was
run with, and the reference output ``x + attention(x, mask, causal)`` (the
layer plus the block residual, torch_transformer_benchmark.py:140), all fp32
on the CPU.  The oracle package is checked against these in
tests/test_oracle.py.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


# (name, batch, seq, d_model, heads, causal, padding_ratio, seed)
ATTENTION_CASES = [
    ("cfg1_noncausal", 2, 128, 256, 4, False, 0.0, 1234),   # benchmark configuration 1 shape
    ("cfg1_causal", 2, 128, 256, 4, True, 0.0, 1235),
    ("padded_causal", 3, 96, 128, 2, True, 0.4, 1236),       # prefix key-padding masks
    ("ragged_hd128", 1, 77, 256, 2, False, 0.3, 1237),       # S not a tile multiple, hd 128
    ("tiny_s1", 2, 1, 64, 1, True, 0.0, 1238),               # single-token sequences
]


def make_attention_fixture(ref, name, B, S, D, H, causal, padding, seed):
    torch.manual_seed(seed)
    layer = ref.BaselineSelfAttention(D, H)
    # Seeded N(0, 0.02) weights (the benchmark configurations' init) loaded through the
    # same strict load_state_dict path the benchmark uses.
    g = torch.Generator().manual_seed(seed + 7)
    sd = {k: torch.randn(v.shape, generator=g) * 0.02 for k, v in layer.state_dict().items()}
    layer.load_state_dict(sd, strict=True)
    layer.eval()
    cfg = ref.TransformerConfig(batch_size=B, seq_len=S, d_model=D, num_heads=H,
                                ffn_dim=4 * D, num_layers=1, causal=causal)
    cfg.validate()
    x, mask = ref.generate_random_case(cfg, torch.device("cpu"), torch.float32, seed,
                                       padding, 1.0)
    with torch.inference_mode():
        out = x + layer(x, mask if padding > 0 else None, causal)
    return {
        "name": name, "batch": B, "seq_len": S, "d_model": D, "heads": H,
        "causal": causal, "padding_ratio": padding, "seed": seed,
        "x": x.clone(), "mask": mask.clone(), "use_mask": padding > 0,
        "state_dict": {k: v.clone() for k, v in sd.items()},
        "out": out.clone(),
    }


def make_block_fixture(ref, seed=2024):
    """A 2-layer BaselineTransformer (the whole reference model) on a small shape."""
    cfg = ref.TransformerConfig(batch_size=2, seq_len=96, d_model=128, num_heads=2, ffn_dim=256,
                                num_layers=2, causal=True)
    torch.manual_seed(seed)
    model = ref.BaselineTransformer(cfg).eval()
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for k, v in model.state_dict().items():
        if k.endswith("norm1.weight") or k.endswith("norm2.weight") or k == "final_norm.weight":
            sd[k] = 1.0 + 0.1 * torch.randn(v.shape, generator=g)
        else:
            sd[k] = torch.randn(v.shape, generator=g) * 0.05
    model.load_state_dict(sd, strict=True)
    x, mask = ref.generate_random_case(cfg, torch.device("cpu"), torch.float32, seed, 0.25, 1.0)
    with torch.inference_mode():
        out = model(x, mask)
    return {"config": dict(batch_size=2, seq_len=96, d_model=128, num_heads=2, ffn_dim=256,
                           num_layers=2, causal=True),
            "x": x, "mask": mask, "state_dict": sd, "out": out}


def make_int8_fixture(k8, seed=4321, tokens=64, d_in=256, d_out=192):
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(d_in, d_out)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(d_out, d_in, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(d_out, generator=g) * 0.02)
        lin.weight[3].zero_()           # exercises the 1e-8 weight-scale clamp
    h = torch.randn(tokens, d_in, generator=g)
    h[5].zero_()                        # exercises the 1e-6 activation-scale clamp
    h[7] *= 1e-3
    a8, s_a = k8._quant_rows(h)
    w_t, s_w, b = k8._int8_pack(lin)
    y = k8._int8_linear(h, w_t, s_w, b)
    acc = torch._int_mm(a8, w_t)
    return {
        "h": h, "weight": lin.weight.detach().clone(), "bias": lin.bias.detach().clone(),
        "a8": a8, "s_a": s_a.view(-1), "w8": w_t.t().contiguous(), "s_w": s_w,
        "acc": acc, "y": y,
    }


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TTJ_REFERENCE_ROOT"),
                    help="path of the reference repository checkout")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or TTJ_REFERENCE_ROOT) is required")
    root = Path(args.reference)
    ref = _load(root / "torch_transformer_benchmark.py", "ttj_reference_benchmark")
    k8 = _load(root / "Project" / "kernels" / "k008_int8_gemm.py", "ttj_reference_k008")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for case in ATTENTION_CASES:
        fx = make_attention_fixture(ref, *case)
        torch.save(fx, HERE / f"attn_{case[0]}.pt")
        print("wrote", f"attn_{case[0]}.pt", tuple(fx["out"].shape))
    fx = make_block_fixture(ref)
    torch.save(fx, HERE / "block_model.pt")
    print("wrote block_model.pt", tuple(fx["out"].shape))
    fx = make_int8_fixture(k8)
    torch.save(fx, HERE / "int8_recipe.pt")
    print("wrote int8_recipe.pt", tuple(fx["acc"].shape))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
