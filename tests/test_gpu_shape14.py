"""Official shape 14 of the reference (Project/shapes.json: B32 S100000 D1024
H16, 2 layers, ffn 1024, causal; the benchmark's default fp32 model) through
the drop-in model ``plugin.build(otb, config)``, evaluated the way the
reference's own long-context evaluation does it
(Project/tools/shape14_eval.py:411-520): B=1 slices drawn from the CUDA
generator with seed ``base_seed * 1000 + batch_index``, each slice's whole
output [1, 100000, 1024] compared with the streamed fp32 model
(``oracle.block_ref.streamed_model_ref``, gated against the dense model in
tests/test_oracle.py) under the reference predicate, with its error
statistics (violations, max and mean absolute error).

Seven base seeds (1234-1240), two slices each; the reference evaluates all 32
slices of five seeds, and slices are independent batch rows.  The reference's
batch-decomposition check (shape14_eval.py:674-751) is restated as: four
slices in one B=4 call equal the four B=1 calls bit for bit.
"""

import types

import pytest
import torch

from oracle import compare_outputs, generate_case
from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef, streamed_model_ref
from tiktok_techjam_2026_track3_b200 import plugin
from tiktok_techjam_2026_track3_b200.config import OFFICIAL_SHAPES

pytestmark = pytest.mark.gpu

SHAPE = OFFICIAL_SHAPES[14]
SEEDS = list(range(1234, 1241))


@pytest.fixture(scope="module")
def models():
    cfg = TransformerConfigRef(batch_size=SHAPE.batch, seq_len=SHAPE.seq_len, d_model=SHAPE.d_model,
                               num_heads=SHAPE.num_heads, ffn_dim=SHAPE.ffn_dim,
                               num_layers=SHAPE.num_layers, causal=SHAPE.causal)
    torch.manual_seed(1234)  # default nn.Linear / nn.LayerNorm init, as the reference's template model
    ref = BaselineTransformerRef(cfg).eval()
    model = plugin.build(types.SimpleNamespace(BaselineTransformer=BaselineTransformerRef), cfg)
    model.load_state_dict(ref.state_dict(), strict=True)
    yield ref.cuda(), model.cuda().eval()
    torch.cuda.empty_cache()


def _slice(base_seed, batch_index):
    x, mask = generate_case(1, SHAPE.seq_len, SHAPE.d_model, base_seed * 1000 + batch_index, device="cuda")
    return x, mask


@pytest.mark.parametrize("seed", SEEDS)
def test_shape14_slices_against_streamed_model(models, seed):
    ref, model = models
    for batch_index in sorted({(seed - 1234) * 4 % 32, ((seed - 1234) * 4 + 17) % 32}):
        x, mask = _slice(seed, batch_index)
        x_before = x.clone()
        with torch.inference_mode():
            out = model(x, mask)
            target = streamed_model_ref(ref, x, mask)
        assert torch.equal(x, x_before)  # the input is not modified
        rep = compare_outputs(target, out)
        print(f"shape 14 seed {seed} slice {batch_index}: {rep}")
        assert rep.passed, f"seed {seed} slice {batch_index}: {rep}"
        del out, target, x, x_before
        torch.cuda.empty_cache()


def test_shape14_batch_decomposition(models):
    _, model = models
    xs = [_slice(1234, b)[0] for b in range(4)]
    with torch.inference_mode():
        whole = model(torch.cat(xs), None)
        for b, x in enumerate(xs):
            assert torch.equal(whole[b:b + 1], model(x, None)), f"row {b}"
