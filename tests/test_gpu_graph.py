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


@pytest.mark.parametrize("sid,dtype", [(2, torch.float32), (7, torch.float16), (8, torch.bfloat16),
                                       (12, torch.float32)])
def test_plugin_model_graph_replay_equals_eager(sid, dtype):
    """The drop-in model replays a captured CUDA graph from the second call with
    the same shape / mask presence / weights on (the reference route's behaviour,
    dispatcher_region.py:1220-1260).  Every call must equal an eager call of the
    same model bit for bit, return a fresh tensor, follow new inputs and masks,
    and pick up new weights."""
    import types
    from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef
    from tiktok_techjam_2026_track3_b200 import plugin
    from tiktok_techjam_2026_track3_b200.config import OFFICIAL_SHAPES
    sh = OFFICIAL_SHAPES[sid]
    B = min(sh.batch, 3)
    cfg = TransformerConfigRef(batch_size=B, seq_len=sh.seq_len, d_model=sh.d_model, num_heads=sh.num_heads,
                               ffn_dim=sh.ffn_dim, num_layers=sh.num_layers, causal=True)
    otb = types.SimpleNamespace(BaselineTransformer=BaselineTransformerRef)
    torch.manual_seed(sid)
    sd = BaselineTransformerRef(cfg).state_dict()
    model = plugin.build(otb, cfg)
    model.load_state_dict(sd)
    model = model.to(device="cuda", dtype=dtype).eval()
    eager = plugin.build(otb, cfg)
    eager.load_state_dict(sd)
    eager = eager.to(device="cuda", dtype=dtype).eval()
    eager.ttj_cuda_graphs = False
    cases = []
    for i, pad in enumerate((0.0, 0.0, 0.0, 0.3, 0.3, 0.3, 0.0)):
        x, m = generate_case(B, cfg.seq_len, cfg.d_model, 4000 + i, dtype=dtype, padding_ratio=pad)
        cases.append((x.cuda(), m.cuda() if pad > 0 else None))
    outs = []
    with torch.inference_mode():
        for x, m in cases:
            out = model(x, m)
            ref = eager(x, m)
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
            assert all(out.data_ptr() != o.data_ptr() for o in outs)
            outs.append(out)
    assert model.__dict__["_ttj_graph_runner"].graph is not None  # replays happened
    # new weights: the next calls follow them (eager, then a new capture)
    sd2 = {k: v * 1.5 for k, v in sd.items()}
    model.load_state_dict(sd2)
    eager.load_state_dict(sd2)
    with torch.inference_mode():
        for x, m in cases[:3]:
            out = model(x, m)
            assert torch.equal(out, eager(x, m))
