"""HostPipeline: host-resident batches with overlapped copies give exactly the
results of calling the layer on each batch in turn."""

import pytest
import torch

from oracle import generate_case, make_weights
from tiktok_techjam_2026_track3_b200 import B200AttentionLayer
from tiktok_techjam_2026_track3_b200.pipeline import HostPipeline

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_pipelined_batches_match_serial_calls(depth):
    B, S, D, H = 2, 512, 1024, 16
    layer = B200AttentionLayer(D, H)
    layer.load_state_dict(make_weights(D, 1234).state_dict())
    layer = layer.to(device="cuda", dtype=torch.float16).eval()
    xs = [generate_case(B, S, D, 1234 + i, dtype=torch.float16)[0].pin_memory() for i in range(5)]
    outs = [torch.empty_like(x).pin_memory() for x in xs]
    pipe = HostPipeline(lambda x: layer(x, None, True), torch.device("cuda", 0), depth=depth)
    with torch.inference_mode():
        pipe.run(xs, outs)
        torch.cuda.synchronize()
        for x, o in zip(xs, outs):
            assert torch.equal(o, layer(x.cuda(), None, True).cpu())
