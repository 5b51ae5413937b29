"""Multi-GPU partitioner for the attention layer: one process per GPU.

Two partitions, both with independent units and therefore no collective in
the compute path (the reference has no multi-GPU code at all; batch rows never
interact, Project/submission/dispatcher_region.py:909-916, and heads never
interact inside attention, dispatcher_region.py:431-434):

* ``"batch"``: rank r owns batch rows ``shard_range(B, world, r)`` and runs the
  whole layer on them.  Optional gather of the output rows to ``dst``.
* ``"heads"`` (single long sequences, B small): every rank holds the whole
  input x; rank r projects only the q/k/v columns of its heads
  ``shard_range(H, world, r)`` and runs attention for them, producing the
  context columns of its heads.  The slices are gathered to ``dst`` with NCCL
  point-to-point receives straight into a K-chunk-major buffer
  ``[world, T, D/world]``, which the out-projection on ``dst`` reads in place
  (``ops.linear_kchunked``), then adds the bias, masks and the residual.
  Sending contexts (T x D/world per rank) moves 4x fewer bytes than reducing
  fp32 partial out-projections (T x D per rank).

The compute steps go through a backend object (default: the CUDA kernels);
tests substitute a CPU backend to exercise the partition and gather logic on
``gloo`` ranks without a GPU.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

__all__ = ["shard_range", "shard_sizes", "CudaBackend", "ShardedAttention"]


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous balanced split of n units: the first n % world ranks get one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_sizes(n: int, world: int) -> List[int]:
    return [shard_range(n, world, r)[1] - shard_range(n, world, r)[0] for r in range(world)]


class CudaBackend:
    """Compute steps on the sm_100a kernels (the product path)."""

    def layer(self, layer, x, mask, causal):
        return layer.forward_residual(x, x, mask, causal)

    def head_context(self, x, w_qkv_r, b_qkv_r, heads_r, causal, mask, out=None):
        from . import ops
        B, S, D = x.shape
        qkv = ops.linear(x.reshape(B * S, D), w_qkv_r, b_qkv_r).view(B, S, w_qkv_r.shape[0])
        return ops.flash_attn(qkv, heads_r, causal, key_mask=mask, out=out)

    def out_proj_chunked(self, ctx_chunks, w_o, b_o, residual, mask):
        from . import ops
        B, S, D = residual.shape
        rm = None if mask is None else mask.reshape(-1)
        return ops.linear_kchunked(ctx_chunks, w_o, b_o, residual=residual.reshape(B * S, D),
                                   row_mask=rm).view(B, S, D)


class ShardedAttention:
    """``x + attention(x)`` partitioned over the ranks of a process group.

    batch mode: ``forward(x_local, ...)`` takes this rank's batch rows
    (``shard_range(global_batch, world, rank)``) and returns its output rows;
    with ``gather=True`` rank ``dst`` returns the full [B,S,D] output.
    heads mode: ``forward(x, ...)`` takes the whole input on every rank and
    returns the full output on ``dst`` (``None`` elsewhere)."""

    def __init__(self, layer, mode: str = "batch", group=None, dst: int = 0, backend=None):
        if mode not in ("batch", "heads"):
            raise ValueError("mode must be 'batch' or 'heads'")
        self.layer = layer
        self.mode = mode
        self.group = group
        self.dst = dst
        self.backend = backend if backend is not None else CudaBackend()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._head_pack = None
        if mode == "heads":
            H = layer.num_heads
            if H % self.world != 0:
                raise ValueError(f"heads ({H}) must divide evenly over {self.world} ranks")

    def _peer(self, r: int) -> int:
        """Global rank of rank ``r`` of this partition's group (``P2POp`` takes
        global ranks; the partition works in group ranks)."""
        return r if self.group is None else dist.get_global_rank(self.group, r)

    # ---------------------------------------------------------------- heads
    def head_weights(self):
        """This rank's slice of the packed projection: q, k and v rows of its heads.

        Cached on the packed weights it was cut from: the layer repacks them
        (new tensors) after ``load_state_dict``, ``.to()`` or an in-place edit,
        and the slice is then cut again."""
        w_qkv, b_qkv, w_o, b_o = self.layer.packed_weights()
        if self._head_pack is None or self._head_pack[0] is not w_qkv or self._head_pack[1] is not b_qkv:
            D = self.layer.d_model
            hd = self.layer.head_dim
            h0, h1 = shard_range(self.layer.num_heads, self.world, self.rank)
            rows = torch.cat([torch.arange(s * D + h0 * hd, s * D + h1 * hd) for s in range(3)])
            rows = rows.to(w_qkv.device)
            self._head_pack = (w_qkv, b_qkv, (w_qkv.index_select(0, rows).contiguous(),
                                              b_qkv.index_select(0, rows).contiguous(), h1 - h0, w_o, b_o))
        return self._head_pack[2]

    def _forward_heads(self, x, mask, causal):
        B, S, D = x.shape
        T = B * S
        w_r, b_r, heads_r, w_o, b_o = self.head_weights()
        dr = heads_r * self.layer.head_dim
        if self.rank == self.dst:
            chunks = torch.empty(self.world, T, dr, dtype=x.dtype, device=x.device)
            self.backend.head_context(x, w_r, b_r, heads_r, causal, mask,
                                      out=chunks[self.rank].view(B, S, dr))
            ops_ = [dist.P2POp(dist.irecv, chunks[r], self._peer(r), group=self.group)
                    for r in range(self.world) if r != self.dst]
            for req in (dist.batch_isend_irecv(ops_) if ops_ else []):
                req.wait()
            return self.backend.out_proj_chunked(chunks, w_o, b_o, x, mask)
        ctx = self.backend.head_context(x, w_r, b_r, heads_r, causal, mask).reshape(T, dr).contiguous()
        for req in dist.batch_isend_irecv([dist.P2POp(dist.isend, ctx, self._peer(self.dst), group=self.group)]):
            req.wait()
        return None

    # ---------------------------------------------------------------- batch
    def _gather_rows(self, local, global_batch):
        sizes = shard_sizes(global_batch, self.world)
        if self.rank == self.dst:
            out = torch.empty(global_batch, *local.shape[1:], dtype=local.dtype, device=local.device)
            starts = [shard_range(global_batch, self.world, r)[0] for r in range(self.world)]
            out[starts[self.rank]:starts[self.rank] + sizes[self.rank]].copy_(local)
            ops_ = [dist.P2POp(dist.irecv, out[starts[r]:starts[r] + sizes[r]], self._peer(r), group=self.group)
                    for r in range(self.world) if r != self.dst and sizes[r] > 0]
            for req in (dist.batch_isend_irecv(ops_) if ops_ else []):
                req.wait()
            return out
        if sizes[self.rank] > 0:
            for req in dist.batch_isend_irecv([dist.P2POp(dist.isend, local.contiguous(), self._peer(self.dst),
                                                          group=self.group)]):
                req.wait()
        return None

    def forward(self, x, valid_token_mask=None, causal=False, gather=True,
                global_batch: Optional[int] = None):
        if self.mode == "heads":
            return self._forward_heads(x, valid_token_mask, causal)
        if x.shape[0] == 0:  # more ranks than batch rows: nothing to compute here
            out = x.new_empty(x.shape)
        else:
            out = self.backend.layer(self.layer, x, valid_token_mask, causal)
        if not gather:
            return out
        if global_batch is None:
            raise ValueError("batch mode gather needs global_batch")
        return self._gather_rows(out, global_batch)

    __call__ = forward
