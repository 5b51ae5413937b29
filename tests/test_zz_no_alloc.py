"""The no-allocation attention-layer entry point, for callers that cannot
allocate device memory (a host runtime that owns every device allocation, or
one that must not grow its footprint after start-up).

ttj_attn_layer_fwd_noalloc keeps the layer's qkv / context intermediates in a
fixed 32 MiB array owned by the library instead of a caller workspace.  It is
called here through the C ABI and compared with the regular entry point
(ttj_attn_layer_fwd, caller-provided workspace) on two calls in a row, with
different inputs, so leftovers from the first call must not leak into the
second.  Tolerance: the reference predicate (abs 2e-3 OR rel 2e-2) used by
every layer test.  The file is named to be collected last.
"""

import ctypes as C

import pytest
import torch

from oracle import compare_outputs, generate_case, make_weights
from tiktok_techjam_2026_track3_b200 import B200AttentionLayer, _lib, ops

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT = 32 << 20


def _args(x, pk, out, B, S, D, H, causal, mask=None, residual=None, workspace=None):
    w_qkv, b_qkv, w_o, b_o = pk
    return _lib.AttnLayerArgs(
        x=x.data_ptr(), w_qkv=w_qkv.data_ptr(), b_qkv=b_qkv.data_ptr(), w_o=w_o.data_ptr(),
        b_o=b_o.data_ptr(), valid_token_mask=None if mask is None else mask.data_ptr(),
        residual=None if residual is None else residual.data_ptr(), out=out.data_ptr(),
        workspace=None if workspace is None else workspace.data_ptr(),
        workspace_bytes=0 if workspace is None else workspace.numel(),
        status=ops.status_word(x.device).data_ptr(), batch=B, seq_len=S, d_model=D,
        num_heads=H, causal=int(causal), dtype=0)


@pytest.mark.parametrize("B,S,D,H,causal,padded", [(2, 1024, 1024, 16, True, False),
                                                   (3, 333, 512, 4, False, True)])
def test_noalloc_matches_regular_entry_point_twice(B, S, D, H, causal, padded):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.ttj_attn_layer_workspace_size(B, S, D, 0) <= SCRATCH_LIMIT
    layer = B200AttentionLayer(D, H)
    layer.load_state_dict(make_weights(D, 42).state_dict())
    layer = layer.to(device=dev, dtype=torch.float16).eval()
    pk = layer.packed_weights()
    for call, seed in enumerate((1234, 1235)):
        x, mask = generate_case(B, S, D, seed, dtype=torch.float16,
                                padding_ratio=0.3 if padded else 0.0)
        x = x.to(dev)
        m8 = mask.to(dev).view(torch.uint8) if padded else None
        out_regular = torch.empty_like(x)
        ws = torch.empty(lib.ttj_attn_layer_workspace_size(B, S, D, 0), dtype=torch.uint8, device=dev)
        a = _args(x, pk, out_regular, B, S, D, H, causal, m8, x, ws)
        assert lib.ttj_attn_layer_fwd(C.byref(a), stream) == 0
        out_noalloc = torch.full_like(x, float("nan"))
        a2 = _args(x, pk, out_noalloc, B, S, D, H, causal, m8, x, None)
        rc = lib.ttj_attn_layer_fwd_noalloc(C.byref(a2), stream)
        assert rc == 0, lib.ttj_last_error()
        torch.cuda.synchronize(dev)
        ops.check_device_status(dev)
        rep = compare_outputs(out_regular.float(), out_noalloc.float())
        assert rep.passed, f"call {call}: {rep}"
        print(f"call {call}: {rep}; bit-identical={torch.equal(out_regular, out_noalloc)}")


def test_later_calls_map_no_more_device_memory():
    """The array is mapped when the library's code first reaches the device (the
    first call at the latest); after that a call must not change the device's free
    memory, which is what a caller that reserved the rest of memory relies on."""
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    B, S, D, H = 2, 512, 512, 8
    layer = B200AttentionLayer(D, H)
    layer.load_state_dict(make_weights(D, 7).state_dict())
    layer = layer.to(device=dev, dtype=torch.float16).eval()
    pk = layer.packed_weights()
    x = generate_case(B, S, D, 7, dtype=torch.float16)[0].to(dev)
    out = torch.empty_like(x)
    a = _args(x, pk, out, B, S, D, H, True, None, x, None)
    assert lib.ttj_attn_layer_fwd_noalloc(C.byref(a), stream) == 0, lib.ttj_last_error()
    torch.cuda.synchronize(dev)
    free_after_first = torch.cuda.mem_get_info(dev)[0]
    first = out.clone()
    for _ in range(3):
        assert lib.ttj_attn_layer_fwd_noalloc(C.byref(a), stream) == 0, lib.ttj_last_error()
    torch.cuda.synchronize(dev)
    assert torch.cuda.mem_get_info(dev)[0] == free_after_first
    assert torch.equal(out, first)
    ops.check_device_status(dev)


def test_noalloc_rejects_unsupported_shapes_before_launching():
    """Unsupported head_dim / dtype are rejected by the same checks as the regular
    entry point, before any kernel is launched (the output stays untouched)."""
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    D, H = 512, 1   # head_dim 512 > 256
    x = torch.zeros(1, 8, D, dtype=torch.float16, device=dev)
    pk = tuple(torch.zeros(n, dtype=torch.float16, device=dev) for n in (3 * D * D, 3 * D, D * D, D))
    out = torch.full_like(x, 7.0)
    a = _args(x, pk, out, 1, 8, D, H, True)
    rc = lib.ttj_attn_layer_fwd_noalloc(C.byref(a), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == -2 and b"head_dim" in lib.ttj_last_error()
    a.dtype = 7
    assert lib.ttj_attn_layer_fwd_noalloc(C.byref(a), torch.cuda.current_stream(dev).cuda_stream) == -1
    torch.cuda.synchronize(dev)
    assert bool((out == 7.0).all())


def test_noalloc_rejects_layers_beyond_its_scratch():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    B, S, D, H = 8, 2048, 1024, 16   # needs 128 MiB of scratch
    assert lib.ttj_attn_layer_workspace_size(B, S, D, 0) > SCRATCH_LIMIT
    x = torch.zeros(1, 8, D, dtype=torch.float16, device=dev)  # never read: rejected first
    pk = tuple(torch.zeros(n, dtype=torch.float16, device=dev) for n in (3 * D * D, 3 * D, D * D, D))
    out = torch.empty_like(x)
    a = _args(x, pk, out, B, S, D, H, True)
    rc = lib.ttj_attn_layer_fwd_noalloc(C.byref(a), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == -6
    assert b"scratch" in lib.ttj_last_error()
