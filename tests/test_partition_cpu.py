"""Partitioner logic on CPU: world_size-2 gloo ranks, compute steps replaced by
the fp32 oracle, results compared with the unpartitioned oracle layer."""

import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from oracle import LayerWeights, attention_layer_ref, generate_case, make_weights, split_heads
from tiktok_techjam_2026_track3_b200 import B200AttentionLayer
from tiktok_techjam_2026_track3_b200.partition import ShardedAttention, shard_range, shard_sizes


class OracleBackend:
    """CPU fp32 stand-ins for the three compute steps of the partitioner."""

    def layer(self, layer, x, mask, causal):
        w = LayerWeights.from_state_dict({k: v.detach() for k, v in layer.state_dict().items()})
        return attention_layer_ref(x, w, layer.num_heads, mask, causal)

    def head_context(self, x, w_r, b_r, heads_r, causal, mask, out=None):
        B, S, _ = x.shape
        dr = w_r.shape[0] // 3
        q, k, v = (split_heads(t, heads_r) for t in F.linear(x.float(), w_r.float(), b_r.float()).split(dr, -1))
        s = q @ k.transpose(-1, -2) * (dr // heads_r) ** -0.5
        if causal:
            s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
        if mask is not None:
            s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
        ctx = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B, S, dr)
        if out is not None:
            out.copy_(ctx)
            return out
        return ctx

    def out_proj_chunked(self, chunks, w_o, b_o, residual, mask):
        world, T, dr = chunks.shape
        B, S, D = residual.shape
        ctx = chunks.permute(1, 0, 2).reshape(T, world * dr)  # K-chunk-major -> [T, D]
        out = F.linear(ctx, w_o.float(), b_o.float()).view(B, S, D)
        if mask is not None:
            out = out.masked_fill(~mask[..., None], 0)
        return residual + out


def test_shard_range_covers_exactly():
    for n in (0, 1, 7, 8, 32, 100):
        for world in (1, 2, 3, 8):
            rs = [shard_range(n, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
            sz = shard_sizes(n, world)
            assert max(sz) - min(sz) <= 1 and sum(sz) == n


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    torch.manual_seed(0)
    B, S, D, H = 3, 40, 128, 4
    x, mask = generate_case(B, S, D, 77, padding_ratio=0.3)
    layer = B200AttentionLayer(D, H)
    layer.load_state_dict(make_weights(D, 5).state_dict())
    results = {}
    # batch shards (3 rows over 2 ranks: uneven) with a gather to rank 0
    sh = ShardedAttention(layer, "batch", backend=OracleBackend())
    r0, r1 = shard_range(B, world, rank)
    out = sh(x[r0:r1], mask[r0:r1], True, gather=True, global_batch=B)
    if rank == 0:
        results["batch"] = out
    # head shards (whole input on both ranks) with the K-chunk-major gather
    sh_h = ShardedAttention(layer, "heads", backend=OracleBackend())
    out_h = sh_h(x, mask, True)
    if rank == 0:
        results["heads"] = out_h
    else:
        assert out_h is None
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        torch.save(results, path)


def test_gloo_batch_and_head_partitions_match_unpartitioned():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "res.pt")
        mp.spawn(_worker, args=(world, _free_port(), path), nprocs=world, join=True)
        res = torch.load(path)
    B, S, D, H = 3, 40, 128, 4
    x, mask = generate_case(B, S, D, 77, padding_ratio=0.3)
    ref = attention_layer_ref(x, make_weights(D, 5), H, mask, True)
    torch.testing.assert_close(res["batch"], ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(res["heads"], ref, rtol=1e-5, atol=1e-5)


def _worker_reload_and_subgroup(rank, world, port, path):
    """Heads mode must pick up new weights loaded between two forwards, and both
    partitions must address their peers correctly inside a subgroup whose ranks
    differ from the global ranks (global ranks 1 and 2 of a 3-rank world)."""
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    B, S, D, H = 3, 40, 128, 4
    x, mask = generate_case(B, S, D, 78, padding_ratio=0.3)
    results = {}
    sub = dist.new_group([1, 2])
    if rank in (1, 2):
        layer = B200AttentionLayer(D, H)
        layer.load_state_dict(make_weights(D, 5).state_dict())
        sh = ShardedAttention(layer, "heads", group=sub, backend=OracleBackend())
        first = sh(x, mask, True)
        layer.load_state_dict(make_weights(D, 6).state_dict())   # new weights, same module
        second = sh(x, mask, True)
        gr = dist.get_rank(sub)
        r0, r1 = shard_range(B, 2, gr)
        shb = ShardedAttention(layer, "batch", group=sub, backend=OracleBackend())
        out_b = shb(x[r0:r1], mask[r0:r1], True, gather=True, global_batch=B)
        if gr == 0:
            results = {"first": first, "second": second, "batch": out_b}
        else:
            assert first is None and second is None and out_b is None
    dist.barrier()
    dist.destroy_process_group()
    if rank == 1:
        torch.save(results, path)


def test_gloo_heads_reload_weights_and_subgroup_ranks():
    world = 3
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "res.pt")
        mp.spawn(_worker_reload_and_subgroup, args=(world, _free_port(), path), nprocs=world, join=True)
        res = torch.load(path)
    B, S, D, H = 3, 40, 128, 4
    x, mask = generate_case(B, S, D, 78, padding_ratio=0.3)
    ref1 = attention_layer_ref(x, make_weights(D, 5), H, mask, True)
    ref2 = attention_layer_ref(x, make_weights(D, 6), H, mask, True)
    torch.testing.assert_close(res["first"], ref1, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(res["second"], ref2, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(res["batch"], ref2, rtol=1e-5, atol=1e-5)
