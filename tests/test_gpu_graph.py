"""CUDA-graph capture of the layer (the reference's optimised route captured
whole forwards, Project/submission/dispatcher_region.py:1246-1249).

The launch path may not allocate outside the caller's workspace or synchronise
the host; a captured forward replayed on new input must give exactly what the
eager call gives on that input (same kernels, same order).
"""

import pytest
import torch

from oracle import generate_case, make_weights
from tiktok_techjam_2026_track3_b200 import B200AttentionLayer

pytestmark = pytest.mark.gpu


def _layer(D, H, dtype, quant=None):
    w = make_weights(D, 1234, dtype=torch.float32)
    m = B200AttentionLayer(D, H, quant=quant)
    m.load_state_dict({k: v.clone() for k, v in w.state_dict().items()}, strict=True)
    return m.to(device="cuda", dtype=dtype).eval()


@pytest.mark.parametrize("quant,dtype,D,H", [(None, torch.float16, 1024, 16),
                                             (None, torch.bfloat16, 1024, 8),
                                             ("int8", torch.bfloat16, 1024, 8)])
@pytest.mark.parametrize("masked", [False, True])
def test_captured_forward_replays_exactly(quant, dtype, D, H, masked):
    B, S = 2, 640
    layer = _layer(D, H, dtype, quant)
    x0, _ = generate_case(B, S, D, 1235, dtype=dtype)
    x1, _ = generate_case(B, S, D, 1236, dtype=dtype)
    mask = None
    if masked:
        mask = torch.ones(B, S, dtype=torch.bool)
        mask[1, 500:] = False
        mask = mask.cuda()
    static_x = x0.cuda()
    with torch.inference_mode():
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):  # warm-up: packs weights, creates the status word
                layer(static_x, mask, True)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_out = layer(static_x, mask, True)
        for x in (x1, x0):
            static_x.copy_(x.cuda())
            graph.replay()
            eager = layer(x.cuda(), mask, True)
            torch.cuda.synchronize()
            assert torch.equal(static_out, eager)
