"""torchrun worker for the multi-GPU partition test (NCCL, one process per GPU).

Launched by tests/test_gpu_multi.py; rank 0 checks the gathered outputs of the
batch and head partitions against the single-GPU layer and exits non-zero on a
mismatch."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import compare_outputs, generate_case, make_weights  # noqa: E402
from tiktok_techjam_2026_track3_b200 import B200AttentionLayer  # noqa: E402
from tiktok_techjam_2026_track3_b200.partition import ShardedAttention, shard_range  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    ok = True
    for (B, S, D, H, dt, causal, pad) in [(4, 1024, 1024, 16, torch.float16, True, 0.0),
                                          (3, 700, 512, 8, torch.bfloat16, True, 0.3),
                                          (1, 4096, 2048, 16, torch.bfloat16, True, 0.0)]:
        x, mask = generate_case(B, S, D, 1234, dtype=dt, padding_ratio=pad)
        x, mask = x.to(dev), mask.to(dev)
        m = mask if pad > 0 else None
        layer = B200AttentionLayer(D, H)
        layer.load_state_dict(make_weights(D, 7).state_dict())
        layer = layer.to(device=dev, dtype=dt).eval()
        with torch.inference_mode():
            full = layer(x, m, causal)
            r0, r1 = shard_range(B, world, rank)
            out_b = ShardedAttention(layer, "batch")(x[r0:r1].contiguous(),
                                                      None if m is None else m[r0:r1].contiguous(),
                                                      causal, gather=True, global_batch=B)
            out_h = ShardedAttention(layer, "heads")(x, m, causal)
        torch.cuda.synchronize(dev)
        if rank == 0:
            rb = compare_outputs(full.float(), out_b.float())
            rh = compare_outputs(full.float(), out_h.float())
            print(f"B{B} S{S} D{D} H{H} {dt}: batch {rb}; heads {rh}", flush=True)
            ok = ok and rb.passed and rh.passed and torch.equal(full, out_b)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
