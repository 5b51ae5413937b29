#!/usr/bin/env python3
"""Benchmark of the B200 attention-layer forward (x + attention(x)).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

Prints ONE JSON line on rank 0.  A step is one attention-layer forward over
one batch of the workload (benchmark configuration 2 by default: B8 S2048 D1024 H16,
causal, fp16).  Multi-GPU runs (torchrun, one process per GPU) are weak
scaling: every rank runs its own batch of the workload, there is no
collective on the data path, and `value` is the tokens of all ranks divided
by the slowest rank's device time.

`value` is kernel-only throughput with inputs resident in HBM: each step is
the three kernels (QKV GEMM, flash attention, out-proj GEMM with the
residual epilogue) bracketed by CUDA events on the launching stream, and the
L2 is flushed (a 256 MB write) between steps, outside the events.  A second
pass of K steps records events between the kernels too: the per-kernel times
(`kernels_ms`, `roofline`) come from it, and its step time is reported as
`ms_per_step_kernel_events` (the inner events stop each kernel's launch from
overlapping the previous kernel's tail).  `e2e` is
the same metric through the public module call with every step's input copied
in from pinned host memory and its output copied back inside the timed region,
the copies of neighbouring steps overlapping the kernels (HostPipeline);
`e2e.serial_value` is the same with nothing overlapped.
`--impl reference` times the reference algorithm on the host CPU (the fp32
restatement in oracle/), the arm the driver compares against.

`--block` (one GPU, fp16/bf16 configs) times instead one whole pre-norm
transformer block (BaselineTransformerBlock: LayerNorm, attention layer,
LayerNorm, GELU FFN with ffn_dim = --ffn-mult x D) through
ttj_transformer_block_fwd, beside the same block in PyTorch eager ops on the
same GPU (cuBLAS GEMMs, ATen LayerNorm / GELU, SDPA attention) for context.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "attention-layer forward tokens/sec and % of tensor-core roofline at 1/2/4/8 B200"
UNIT = "tokens/s"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2, choices=(2, 3, 4, 5))
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--batch", type=int, default=None, help="override the workload batch")
    ap.add_argument("--seq", type=int, default=None, help="override the workload seq_len")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-seconds", type=float, default=15.0)
    ap.add_argument("--spinup-seconds", type=float, default=0.5,
                    help="untimed work after warm-up so clocks leave idle (0 under a profiler)")
    ap.add_argument("--block", action="store_true",
                    help="time one whole transformer block instead of the attention layer")
    ap.add_argument("--ffn-mult", type=int, default=4, help="ffn_dim = ffn_mult * d_model (--block)")
    ap.add_argument("--shape", type=int, default=None, choices=range(1, 15),
                    help="time an official whole-model shape (Project/shapes.json ids 1-14) instead; "
                         "14 is timed as the reference's long-context evaluation times it")
    ap.add_argument("--dtype", default="float32", choices=("float32", "float16", "bfloat16"),
                    help="model dtype for --shape (the reference benchmark's default is float32)")
    return ap.parse_args()


# --------------------------------------------------------------------- distributed
def init_dist(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML, read
    only, every ~2 ms in a background thread for the duration of the timed
    region (nvidia-smi's process start-up alone is longer than a short timed
    region)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: torch.device):
        self.device = device
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._handle = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            props = torch.cuda.get_device_properties(device)
            bus = getattr(props, "pci_bus_id", None)
            handle = None
            if bus is not None:
                dom = getattr(props, "pci_domain_id", 0)
                dev_id = getattr(props, "pci_device_id", 0)
                try:
                    handle = pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev_id:02x}.0")
                except Exception:
                    handle = None
            if handle is None and pynvml.nvmlDeviceGetCount() == 1:
                handle = pynvml.nvmlDeviceGetHandleByIndex(0)
            self._handle = handle
            if handle is not None:
                self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._handle = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._handle is not None:
            import threading
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = sorted(n for b, n in self.REASONS.items() if bits & b)
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz), "source": "nvml"}


# --------------------------------------------------------------------- peaks
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


def exp_roofline(cfg, attn_ms: float, clocks):
    """The attention's other ceiling: softmax exponentials (one per score the
    reference evaluates: B*H*S^2, B*H*S(S+1)/2 when causal) against the
    exponential unit's 16 results per clock per SM at the sampled SM clock."""
    B, H, S = cfg.batch, cfg.num_heads, cfg.seq_len
    exps = B * H * (S * (S + 1) / 2 if cfg.causal else S * S)
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    peak = 16.0 * sms * mhz * 1e6
    achieved = exps / (attn_ms / 1e3)
    return {"achieved": achieved, "peak": peak, "unit": "exp/s", "frac": achieved / peak,
            "peak_basis": f"16 exp/clk/SM x {sms} SMs x {mhz:.0f} MHz (sampled SM clock)"}


def ncu_traffic(kernel: str, workload: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d.get(workload, {}).get(kernel)


# --------------------------------------------------------------------- CPU arm
def cpu_reference_rate(cfg, seconds: float, seed: int = 1234):
    """Tokens/s of the reference algorithm (fp32, the oracle restatement of
    torch_transformer_benchmark.py:85-122 + :140) on the host CPU, timed with
    perf_counter like the reference's CPU loop (:502-506).

    Up to S = 8192 one step is one dense forward of one batch row (batch rows
    never interact).  Longer sequences cannot be run densely (the score table
    of one row is H*S*S*4 bytes), so one 128-query stripe at the end of the
    sequence (the longest causal key range) of one head is run through the
    streamed oracle and the full-layer time is extrapolated by FLOP ratio;
    the sample string says so."""
    from oracle import attention_layer_ref, attention_layer_streamed_ref, generate_case, make_weights
    from tiktok_techjam_2026_track3_b200.config import attention_flops
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = make_weights(cfg.d_model, seed)
    if cfg.seq_len <= 8192:
        x, _ = generate_case(1, cfg.seq_len, cfg.d_model, seed)
        with torch.inference_mode():
            attention_layer_ref(x, w, cfg.num_heads, None, cfg.causal)  # warm-up
            t0 = time.perf_counter()
            n = 0
            while True:
                attention_layer_ref(x, w, cfg.num_heads, None, cfg.causal)
                n += 1
                el = time.perf_counter() - t0
                if el >= seconds or n >= 200:
                    break
        return (n * cfg.seq_len / el, threads,
                f"{n} forwards of 1 batch row (S={cfg.seq_len}, D={cfg.d_model}, H={cfg.num_heads}, fp32) in {el:.1f}s")
    x, _ = generate_case(1, cfg.seq_len, cfg.d_model, seed)
    rows = torch.arange(cfg.seq_len - 128, cfg.seq_len)
    with torch.inference_mode():
        t0 = time.perf_counter()
        attention_layer_streamed_ref(x, w, cfg.num_heads, cfg.causal, [0], [0], rows, k_chunk=16384)
        el = time.perf_counter() - t0
    hd = cfg.head_dim
    keys = cfg.seq_len  # last rows see every key
    sample_flops = 4.0 * 128 * keys * hd + 2.0 * cfg.seq_len * cfg.d_model * 2 * hd + 2.0 * 128 * cfg.d_model * hd
    full_flops = attention_flops(cfg.with_(batch=1))
    est = el * full_flops / sample_flops
    return (cfg.seq_len / est, threads,
            f"extrapolated: 128-query stripe x 1 head of S={cfg.seq_len} (streamed fp32 oracle, "
            f"{el:.1f}s), scaled by FLOPs to one batch row")


def run_reference(args, cfg):
    """The reference arm: the reference algorithm (the oracle's fp32 restatement
    of BaselineSelfAttention.forward + the block residual, checked against the
    reference's own outputs by tests/test_oracle.py) on the host CPU with every
    thread, on the SAME configuration as our arm.  Up to S = 8192 each step is
    one forward of the whole configured batch (batch rows are evaluated a few at
    a time when their score tables would not fit in host memory; rows never
    interact, so the work and result are the whole batch's).  Longer sequences
    cannot run densely; one step then is the streamed-oracle stripe of
    cpu_reference_rate, extrapolated by FLOPs and labelled so."""
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    if cfg.seq_len > 8192:
        value, threads, sample = cpu_reference_rate(cfg, 10.0)
        line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": 1, "warmup": 0, "ms_per_step": 1e3 * cfg.seq_len / value,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded)", "config": {"workload": cfg.name, "sample": sample},
                "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    from oracle import attention_layer_ref, generate_case, make_weights
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    B, S, D, H = cfg.batch, cfg.seq_len, cfg.d_model, cfg.num_heads
    # score table + probabilities of one batch row: 2 * H * S^2 fp32; keep ~8 GB in flight
    per_row = 2 * H * S * S * 4
    chunk = max(1, min(B, (8 << 30) // per_row))
    x, _ = generate_case(B, S, D, 1234, input_scale=cfg.input_scale)
    w = make_weights(D, 1234)
    per_step = []
    with torch.inference_mode():
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            attention_layer_ref(x, w, H, None, cfg.causal, batch_chunk=chunk)
            el = time.perf_counter() - t0
            if i >= args.warmup:
                per_step.append(el)
    sec = sum(per_step)
    value = B * S * len(per_step) / sec
    sample = (f"every step one whole forward of the configured batch (B={B}, S={S}, D={D}, H={H}, fp32, "
              f"{chunk} batch row(s) at a time), {len(per_step)} timed steps")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sec / len(per_step),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, N(0,1) inputs, N(0,0.02) weights)",
        "config": {"workload": cfg.name, "batch": B, "seq_len": S, "d_model": D, "heads": H,
                   "causal": cfg.causal, "same_config_as_ours": True, "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------- GPU arm
def run_ours_heads(args, cfg, rank, world, local):
    """Config 5 on N GPUs: head-sharded layer (strong scaling), context slices
    gathered to rank 0 over NCCL, out-proj + residual on rank 0."""
    from oracle import make_weights
    from tiktok_techjam_2026_track3_b200 import B200AttentionLayer, ops
    from tiktok_techjam_2026_track3_b200.config import attention_flops
    from tiktok_techjam_2026_track3_b200.partition import ShardedAttention
    import torch.distributed as dist
    dev = torch.device("cuda", local)
    dtype = cfg.torch_dtype
    B, S, D, H = cfg.batch, cfg.seq_len, cfg.d_model, cfg.num_heads
    T = B * S
    layer = B200AttentionLayer(D, H)
    layer.load_state_dict(make_weights(D, 1234).state_dict())
    layer = layer.to(device=dev, dtype=dtype).eval()
    g = torch.Generator(device=dev)
    g.manual_seed(1234)
    x = torch.randn(B, S, D, generator=g, device=dev, dtype=dtype) * cfg.input_scale
    sh = ShardedAttention(layer, "heads")
    w_r, b_r, heads_r, w_o, b_o = sh.head_weights()
    dr = heads_r * layer.head_dim
    stream = torch.cuda.current_stream(dev)
    chunks = torch.empty(world, T, dr, dtype=dtype, device=dev) if rank == 0 else None
    ctx_local = torch.empty(T, dr, dtype=dtype, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step(ev):
        ev[0].record(stream)
        qkv = ops.linear(x.view(T, D), w_r, b_r).view(B, S, 3 * dr)
        ev[1].record(stream)
        dst = (chunks[0] if rank == 0 else ctx_local).view(B, S, dr)
        ops.flash_attn(qkv, heads_r, cfg.causal, out=dst)
        ev[2].record(stream)
        if rank == 0:
            reqs = dist.batch_isend_irecv([dist.P2POp(dist.irecv, chunks[r], r) for r in range(1, world)])
        else:
            reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, ctx_local, 0)])
        for q in reqs:
            q.wait()
        ev[3].record(stream)
        if rank == 0:
            ops.linear_kchunked(chunks, w_o, b_o, residual=x.view(T, D))
        ev[4].record(stream)

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    warm = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    with torch.inference_mode():
        for _ in range(max(1, args.warmup)):
            step(warm)
        torch.cuda.synchronize(dev)
        barrier(world)
        with ClockSampler(dev) as clk:
            for i in range(args.steps):
                flush.zero_()
                barrier(world)
                step(evs[i])
            torch.cuda.synchronize(dev)
        barrier(world)
    ops.check_device_status(dev)
    step_ms = sum(e[0].elapsed_time(e[4]) for e in evs)
    total_ms = max_over_ranks(step_ms, world)
    ms_per_step = total_ms / args.steps
    attn_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    gather_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in evs)
    out_ms = statistics.mean(e[3].elapsed_time(e[4]) for e in evs)
    qkv_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    peaks = measured_peaks()
    flops_attn_r = attention_flops(cfg.with_(num_heads=heads_r, d_model=dr), include_projections=False)
    achieved = flops_attn_r / (attn_ms / 1e3) / 1e12
    layer_tf = attention_flops(cfg) / (ms_per_step / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": T / (ms_per_step / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; x ~ N(0,1), weights/biases ~ N(0,0.02))",
        "config": {"workload": cfg.name, "batch": B, "seq_len": S, "d_model": D, "heads": H,
                   "heads_per_gpu": heads_r, "causal": cfg.causal,
                   "parallelism": f"heads x{world}, NCCL gather of context slices to rank 0",
                   "l2": "flushed between timed steps (256 MB write, outside the events)"},
        "layer_tflops": layer_tf, "layer_frac_of_peak": layer_tf / (world * peaks["bf16_tflops"]),
        "kernels_ms": {"qkv_gemm_rank0": qkv_ms, "flash_attn_rank0": attn_ms, "gather_rank0": gather_ms,
                       "out_proj_residual_rank0": out_ms},
        "roofline": {"kernel": "flash_attn", "bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "peak_source": f"{peaks['source']} (bf16 dense burst)", "traffic": None},
        "gather_gbs": (world - 1) * T * dr * 2 / (gather_ms / 1e3) / 1e9 if rank == 0 else None,
        "gpu_launches": 4 * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_ours_batch_strong(args, cfg, rank, world, local):
    """Configurations 3 and 4 on N GPUs: the configured batch split over the ranks
    (rank r runs rows shard_range(B, N, r) through the layer, strong scaling)
    and every rank's output rows gathered into one [B,S,D] tensor on rank 0
    with NCCL point-to-point receives, inside the timed region
    (ShardedAttention "batch" mode)."""
    from oracle import make_weights
    from tiktok_techjam_2026_track3_b200 import B200AttentionLayer, ops
    from tiktok_techjam_2026_track3_b200.config import attention_flops
    from tiktok_techjam_2026_track3_b200.partition import ShardedAttention, shard_range
    dev = torch.device("cuda", local)
    dtype = cfg.torch_dtype
    B, S, D, H = cfg.batch, cfg.seq_len, cfg.d_model, cfg.num_heads
    r0, r1 = shard_range(B, world, rank)
    layer = B200AttentionLayer(D, H, quant=cfg.quant)
    layer.load_state_dict(make_weights(D, 1234).state_dict())
    layer = layer.to(device=dev, dtype=dtype).eval()
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    x = torch.randn(r1 - r0, S, D, generator=g, device=dev, dtype=dtype) * cfg.input_scale
    sh = ShardedAttention(layer, "batch")
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step(ev):
        ev[0].record(stream)
        out = sh.backend.layer(layer, x, None, cfg.causal)
        ev[1].record(stream)
        sh._gather_rows(out, B)
        ev[2].record(stream)

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    warm = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with torch.inference_mode():
        for _ in range(max(1, args.warmup)):
            step(warm)
        torch.cuda.synchronize(dev)
        barrier(world)
        with ClockSampler(dev) as clk:
            for i in range(args.steps):
                flush.zero_()
                barrier(world)
                step(evs[i])
            torch.cuda.synchronize(dev)
        barrier(world)
    ops.check_device_status(dev)
    total_ms = max_over_ranks(sum(e[0].elapsed_time(e[2]) for e in evs), world)
    ms_per_step = total_ms / args.steps
    layer_ms = max_over_ranks(statistics.mean(e[0].elapsed_time(e[1]) for e in evs), world)
    gather_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    peaks = measured_peaks()
    layer_tf = attention_flops(cfg) / (ms_per_step / 1e3) / 1e12
    rows_max = max(shard_range(B, world, r)[1] - shard_range(B, world, r)[0] for r in range(world))
    local_cfg = cfg.with_(batch=rows_max)
    achieved = attention_flops(local_cfg) / (layer_ms / 1e3) / 1e12
    # the slowest rank's layer against the time its kernels would take at their peaks
    # (int8 projections against twice the bf16 dense peak)
    proj = attention_flops(local_cfg) - attention_flops(local_cfg, include_projections=False)
    peak_gemm = peaks["bf16_tflops"] * (2.0 if cfg.quant == "int8" else 1.0)
    ideal_ms = 1e3 * (proj / (peak_gemm * 1e12)
                      + attention_flops(local_cfg, include_projections=False) / (peaks["bf16_tflops"] * 1e12))
    line = {
        "metric": METRIC, "value": B * S / (ms_per_step / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": {"float16": "fp16", "bfloat16": "bf16"}[cfg.dtype] + ("+int8" if cfg.quant else ""),
        "data": "synthetic (seeded; x ~ N(0,1), weights/biases ~ N(0,0.02))",
        "config": {"workload": cfg.name, "batch": B, "rows_per_gpu": rows_max, "seq_len": S, "d_model": D,
                   "heads": H, "causal": cfg.causal,
                   "parallelism": f"batch split over {world} GPUs, NCCL gather of output rows to rank 0",
                   "l2": "flushed between timed steps (256 MB write, outside the events)"},
        "layer_tflops": layer_tf,
        "layer_frac_of_peak": ideal_ms / layer_ms,
        "kernels_ms": {"layer_slowest_rank": layer_ms, "gather_rank_local": gather_ms},
        "roofline": {"kernel": "attention_layer (slowest rank)", "bound": "tensor", "achieved": achieved,
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": ideal_ms / layer_ms,
                     "peak_source": f"{peaks['source']} (bf16 dense burst; int8 GEMMs against 2x)",
                     "traffic": None},
        "gather_gbs": (B - (r1 - r0)) * S * D * 2 / (gather_ms / 1e3) / 1e9 if rank == 0 and world > 1 else None,
        "gpu_launches": (5 if cfg.quant else 3) * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_ours(args, cfg):
    from oracle import make_weights  # only to seed weights identically to the tests
    from tiktok_techjam_2026_track3_b200 import B200AttentionLayer, ops
    from tiktok_techjam_2026_track3_b200 import _lib
    import ctypes as C

    rank, world, local = init_dist(args.gpus)
    if cfg.shard == "heads" and world > 1:
        rc = run_ours_heads(args, cfg, rank, world, local)
        torch.distributed.destroy_process_group()
        return rc
    if cfg.scaling == "strong" and world > 1:
        rc = run_ours_batch_strong(args, cfg, rank, world, local)
        torch.distributed.destroy_process_group()
        return rc
    dev = torch.device("cuda", local if world > 1 else 0)
    dtype = cfg.torch_dtype
    B, S, D, H = cfg.batch, cfg.seq_len, cfg.d_model, cfg.num_heads
    T = B * S
    layer = B200AttentionLayer(D, H, quant=cfg.quant)
    layer.load_state_dict(make_weights(D, 1234).state_dict())
    layer = layer.to(device=dev, dtype=dtype).eval()
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    x = torch.randn(B, S, D, generator=g, device=dev, dtype=dtype) * cfg.input_scale
    lib = _lib.load()
    dt = 0 if dtype == torch.float16 else 1
    status = ops.status_word(dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    # Pre-allocated buffers: the timed step is exactly the three kernels.
    if cfg.quant == "int8":
        w8, s8, b32, wo8, so8, bo32 = layer.packed_weights()
        act8 = torch.empty(T, D, dtype=torch.int8, device=dev)
        s_tok = torch.empty(T, dtype=torch.float32, device=dev)
    else:
        w_qkv, b_qkv, w_o, b_o = layer.packed_weights()
    qkv = torch.empty(T, 3 * D, dtype=dtype, device=dev)
    ctx = torch.empty(T, D, dtype=dtype, device=dev)
    out = torch.empty_like(x)

    def step(ev):
        # ev: 4 events (step start, after the QKV projection, after attention,
        # step end) or 2 (step start and end only: nothing between the kernels,
        # so each overlaps the previous one's tail as in a user's stream).
        inner = len(ev) == 4
        rc = 0
        ev[0].record(stream)
        if cfg.quant == "int8":
            rc |= lib.ttj_int8_quant_rows(x.data_ptr(), act8.data_ptr(), s_tok.data_ptr(), T, D, dt, sp)
            rc |= lib.ttj_int8_linear_fwd(act8.data_ptr(), s_tok.data_ptr(), w8.data_ptr(), s8.data_ptr(),
                                          b32.data_ptr(), None, None, qkv.data_ptr(), T, 3 * D, D, dt,
                                          status.data_ptr(), sp)
        else:
            rc |= lib.ttj_qkv_proj_fwd(x.data_ptr(), w_qkv.data_ptr(), b_qkv.data_ptr(), qkv.data_ptr(),
                                       T, D, dt, status.data_ptr(), sp)
        if inner:
            ev[1].record(stream)
        rc |= lib.ttj_flash_attn_fwd(qkv.data_ptr(), None, ctx.data_ptr(), B, S, H, D // H,
                                     int(cfg.causal), dt, status.data_ptr(), sp)
        if inner:
            ev[2].record(stream)
        if cfg.quant == "int8":
            rc |= lib.ttj_int8_quant_rows(ctx.data_ptr(), act8.data_ptr(), s_tok.data_ptr(), T, D, dt, sp)
            rc |= lib.ttj_int8_linear_fwd(act8.data_ptr(), s_tok.data_ptr(), wo8.data_ptr(), so8.data_ptr(),
                                          bo32.data_ptr(), x.data_ptr(), None, out.data_ptr(), T, D, D, dt,
                                          status.data_ptr(), sp)
        else:
            rc |= lib.ttj_out_proj_residual_fwd(ctx.data_ptr(), w_o.data_ptr(), b_o.data_ptr(), x.data_ptr(),
                                                None, out.data_ptr(), T, D, dt, status.data_ptr(), sp)
        ev[-1].record(stream)
        if rc:
            raise RuntimeError(f"launch failed: {lib.ttj_last_error().decode()}")

    launches_per_step = 5 if cfg.quant == "int8" else 3
    # Two timed passes of K steps each: the first with events at step
    # boundaries only (`value`), the second with events between the kernels
    # (per-kernel times for the roofline; those events keep the kernels of a
    # step from overlapping, so this pass runs slightly slower).
    step_evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    warm = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    with torch.inference_mode():
        for _ in range(args.warmup):
            flush.zero_()
            step(warm)
        # Untimed spin-up so SM clocks have left idle before timing starts.
        t_spin = time.perf_counter()
        while time.perf_counter() - t_spin < args.spinup_seconds:
            for _ in range(20):
                step(warm)
            torch.cuda.synchronize(dev)
        torch.cuda.synchronize(dev)
        barrier(world)
        torch.cuda.synchronize(dev)
        with ClockSampler(dev) as clk:
            for i in range(args.steps):
                flush.zero_()
                step(step_evs[i])
            for i in range(args.steps):
                flush.zero_()
                step(evs[i])
            torch.cuda.synchronize(dev)
        barrier(world)
        torch.cuda.synchronize(dev)
    ops.check_device_status(dev)
    step_ms = [e[0].elapsed_time(e[1]) for e in step_evs]
    step_ms_split = [e[0].elapsed_time(e[3]) for e in evs]
    qkv_ms = [e[0].elapsed_time(e[1]) for e in evs]
    attn_ms = [e[1].elapsed_time(e[2]) for e in evs]
    outp_ms = [e[2].elapsed_time(e[3]) for e in evs]
    total_ms = max_over_ranks(sum(step_ms), world)
    ms_per_step = total_ms / args.steps
    value = world * T * args.steps / (total_ms / 1e3)

    # ---- roofline of the dominant kernel (largest share of the step)
    from tiktok_techjam_2026_track3_b200.config import attention_flops
    peaks = measured_peaks()
    flops_attn = attention_flops(cfg, include_projections=False)
    flops_qkv = 2.0 * T * D * 3 * D
    flops_out = 2.0 * T * D * D
    # Each kernel against the peak of its own arithmetic: the int8 projections
    # against twice the bf16 dense peak, attention (16-bit) against the bf16 peak.
    peak_bf16 = peaks["bf16_tflops"]
    peak_gemm = peak_bf16 * (2.0 if cfg.quant == "int8" else 1.0)
    kernels = {
        "qkv_gemm": (statistics.mean(qkv_ms), flops_qkv, peak_gemm),
        "flash_attn": (statistics.mean(attn_ms), flops_attn, peak_bf16),
        "out_proj_residual": (statistics.mean(outp_ms), flops_out, peak_gemm),
    }
    dom = max(kernels, key=lambda k: kernels[k][0])
    dom_ms, dom_flops, peak_tf = kernels[dom]
    achieved = dom_flops / (dom_ms / 1e3) / 1e12
    layer_tf = attention_flops(cfg) / (ms_per_step / 1e3) / 1e12
    # The layer's fraction of its roofline: the time every kernel would take at
    # its peak, over the measured step time.
    ideal_ms = sum(fl / (pk * 1e12) * 1e3 for _, fl, pk in kernels.values())
    clocks = clk.summary()

    # ---- e2e through the public module call, pinned host buffers allocated in
    # memory local to this GPU's NUMA node
    from tiktok_techjam_2026_track3_b200.pipeline import HostPipeline, near_device
    with near_device(dev) as local_cpus:
        x_host = x.cpu().pin_memory()
        out_host = torch.empty(x_host.shape, dtype=dtype).pin_memory()
        outs_host = [torch.empty(x_host.shape, dtype=dtype).pin_memory() for _ in range(2)]
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    with torch.inference_mode():
        for _ in range(max(3, args.warmup)):
            out_host.copy_(layer(x_host.to(dev, non_blocking=True), None, cfg.causal), non_blocking=True)
        torch.cuda.synchronize(dev)
        barrier(world)
        for i in range(args.steps):
            flush.zero_()
            e2e_ev[i][0].record(stream)
            xd = x_host.to(dev, non_blocking=True)
            o = layer(xd, None, cfg.causal)
            out_host.copy_(o, non_blocking=True)
            e2e_ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
    e2e_serial_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in e2e_ev), world)
    e2e_serial = world * T * args.steps / (e2e_serial_ms / 1e3)
    nbytes = x_host.numel() * x_host.element_size()

    # ---- e2e pipelined across steps (HostPipeline): step i+1's input copy and
    # step i-1's output copy overlap step i's kernels.  Every step still copies
    # its input in from pinned host memory and its result back.  No L2 flush:
    # each step streams ~200 MB (input, qkv, ctx, output), more than the L2.
    pipe = HostPipeline(lambda xd: layer(xd, None, cfg.causal), dev, depth=2)
    with torch.inference_mode():
        pipe.run([x_host] * max(3, args.warmup), [outs_host[i % 2] for i in range(max(3, args.warmup))])
        torch.cuda.synchronize(dev)
        barrier(world)
        torch.cuda.synchronize(dev)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        pipe.run([x_host] * args.steps, [outs_host[i % 2] for i in range(args.steps)])
        p1.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
    e2e_ms = max_over_ranks(p0.elapsed_time(p1), world)
    e2e_value = world * T * args.steps / (e2e_ms / 1e3)

    # ---- the host link's ceiling for the e2e leg on this box: the same two
    # copies per step (input in, output back, from the same pinned buffers)
    # issued on two streams with nothing else queued, so both directions run at
    # once; ceiling = tokens per step / the time a step of copies takes.
    n_copy = max(args.steps, 20)
    xs_dev = torch.empty(x_host.shape, dtype=dtype, device=dev)
    ys_dev = torch.empty(x_host.shape, dtype=dtype, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    for s_ in (s_in, s_out):
        s_.wait_stream(stream)
    with torch.cuda.stream(s_in):
        xs_dev.copy_(x_host, non_blocking=True)
    with torch.cuda.stream(s_out):
        outs_host[0].copy_(ys_dev, non_blocking=True)
    torch.cuda.synchronize(dev)
    barrier(world)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    for s_ in (s_in, s_out):
        s_.wait_stream(stream)
    for i in range(n_copy):
        with torch.cuda.stream(s_in):
            xs_dev.copy_(x_host, non_blocking=True)
        with torch.cuda.stream(s_out):
            outs_host[i % 2].copy_(ys_dev, non_blocking=True)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    c1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    copies_ms = max_over_ranks(c0.elapsed_time(c1), world)
    copies_value = world * T * n_copy / (copies_ms / 1e3)
    del xs_dev, ys_dev

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": {"float16": "fp16", "bfloat16": "bf16"}[cfg.dtype] + ("+int8" if cfg.quant else ""),
        "data": "synthetic (seeded; x ~ N(0,1), weights/biases ~ N(0,0.02))",
        "config": {"workload": cfg.name, "batch_per_gpu": B, "seq_len": S, "d_model": D,
                   "heads": H, "head_dim": D // H, "causal": cfg.causal, "parallelism": f"dp{world} (batch shards, weak)",
                   "l2": "flushed between timed steps (256 MB write, outside the events)"},
        "layer_tflops": layer_tf,
        "layer_frac_of_peak": ideal_ms / ms_per_step,
        "kernels_ms": {k: v[0] for k, v in kernels.items()},
        "ms_per_step_kernel_events": statistics.mean(step_ms_split),
        "roofline": {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": peak_tf,
                     "unit": "TFLOP/s", "frac": achieved / peak_tf,
                     "peak_source": f"{peaks['source']} ({'2x ' if cfg.quant and dom != 'flash_attn' else ''}bf16 dense burst)",
                     "traffic": ncu_traffic(dom, cfg.name),
                     "exp_unit": exp_roofline(cfg, statistics.mean(attn_ms), clocks)},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": nbytes,
                "d2h_bytes_per_step": nbytes,
                "mode": "B200AttentionLayer calls through HostPipeline (copies of steps i+1 / i-1 overlap step i)",
                "serial_value": e2e_serial,
                "copies_only_value": copies_value,
                "copies_only": "one step's input copy in and output copy back on two streams, nothing else queued",
                "frac_of_copies_only": e2e_value / copies_value,
                "pinned_near_cpus": None if local_cpus is None else f"{len(local_cpus)} CPUs ({local_cpus[0]}-{local_cpus[-1]})"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_reference_rate(cfg, args.cpu_sample_seconds)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def run_block(args, cfg):
    """One transformer block per step through ttj_transformer_block_fwd (see the
    module docstring), with the PyTorch eager block timed beside it."""
    import ctypes as C
    import torch.nn.functional as F
    from tiktok_techjam_2026_track3_b200 import _lib, ops

    if args.gpus != 1 or cfg.quant is not None:
        raise SystemExit("--block runs on one GPU with a 16-bit config")
    dev = torch.device("cuda", 0)
    dtype = cfg.torch_dtype
    B, S, D, H = cfg.batch, cfg.seq_len, cfg.d_model, cfg.num_heads
    Fd = args.ffn_mult * D
    T = B * S
    g = torch.Generator(device=dev)
    g.manual_seed(1234)

    def rnd(*shape, scale=0.02, offset=0.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale + offset).to(dtype)

    prm = {"ln1_w": rnd(D, offset=1.0), "ln1_b": rnd(D), "w_qkv": rnd(3 * D, D), "b_qkv": rnd(3 * D),
           "w_o": rnd(D, D), "b_o": rnd(D), "ln2_w": rnd(D, offset=1.0), "ln2_b": rnd(D),
           "w_in": rnd(Fd, D), "b_in": rnd(Fd), "w_out": rnd(D, Fd), "b_out": rnd(D)}
    x = rnd(B, S, D, scale=1.0)
    out = torch.empty_like(x)
    lib = _lib.load()
    dt = 0 if dtype == torch.float16 else 1
    ws = torch.empty(lib.ttj_block_workspace_size(B, S, D, Fd, dt), dtype=torch.uint8, device=dev)
    status = ops.status_word(dev)
    stream = torch.cuda.current_stream(dev)
    a = _lib.BlockArgs(x=x.data_ptr(), valid_token_mask=None, out=out.data_ptr(),
                       workspace=ws.data_ptr(), workspace_bytes=ws.numel(), status=status.data_ptr(),
                       batch=B, seq_len=S, d_model=D, num_heads=H, ffn_dim=Fd, eps1=1e-5, eps2=1e-5,
                       causal=int(cfg.causal), dtype=dt, **{k: v.data_ptr() for k, v in prm.items()})

    def ours():
        rc = lib.ttj_transformer_block_fwd(C.byref(a), stream.cuda_stream)
        if rc:
            raise RuntimeError(lib.ttj_last_error().decode())

    # The same block given an all-true valid_token_mask, as the reference's
    # benchmark passes for unpadded inputs (torch_transformer_benchmark.py:255-259).
    ones = torch.ones(B, S, dtype=torch.uint8, device=dev)
    out_m = torch.empty_like(out)
    a_m = _lib.BlockArgs(**{f: getattr(a, f) for f, _ in _lib.BlockArgs._fields_})
    a_m.valid_token_mask = ones.data_ptr()
    a_m.out = out_m.data_ptr()

    def ours_masked():
        rc = lib.ttj_transformer_block_fwd(C.byref(a_m), stream.cuda_stream)
        if rc:
            raise RuntimeError(lib.ttj_last_error().decode())

    def torch_eager():
        h = F.layer_norm(x, (D,), prm["ln1_w"], prm["ln1_b"], 1e-5)
        q, k, v = F.linear(h, prm["w_qkv"], prm["b_qkv"]).view(B, S, 3, H, D // H).permute(2, 0, 3, 1, 4)
        c = F.scaled_dot_product_attention(q, k, v, is_causal=cfg.causal).transpose(1, 2).reshape(B, S, D)
        x1 = x + F.linear(c, prm["w_o"], prm["b_o"])
        h2 = F.layer_norm(x1, (D,), prm["ln2_w"], prm["ln2_b"], 1e-5)
        return x1 + F.linear(F.gelu(F.linear(h2, prm["w_in"], prm["b_in"])), prm["w_out"], prm["b_out"])

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def time_it(fn):
        with torch.inference_mode():
            for _ in range(args.warmup):
                fn()
            t_spin = time.perf_counter()
            while time.perf_counter() - t_spin < args.spinup_seconds:
                fn()
                torch.cuda.synchronize(dev)
            ms = []
            for _ in range(args.steps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                torch.cuda.synchronize(dev)
                ms.append(e0.elapsed_time(e1))
        return sum(ms) / len(ms)

    with ClockSampler(dev) as clk:
        ours_ms = time_it(ours)
    masked_ms = time_it(ours_masked)
    torch_ms = time_it(torch_eager)
    ops.check_device_status(dev)
    with torch.inference_mode():
        err = float((out.float() - torch_eager().float()).abs().max())
    from tiktok_techjam_2026_track3_b200.config import attention_flops
    flops = attention_flops(cfg) + 2.0 * 2 * T * D * Fd
    line = {
        "metric": "transformer-block forward tokens/sec", "value": T / (ours_ms / 1e3), "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ours_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {"float16": "fp16", "bfloat16": "bf16"}[cfg.dtype],
        "data": "synthetic (seeded; x ~ N(0,1), weights ~ N(0,0.02), norm weights ~ 1 + N(0,0.02))",
        "config": {"workload": f"block_{cfg.name}_ffn{Fd}", "batch": B, "seq_len": S, "d_model": D,
                   "heads": H, "ffn_dim": Fd, "causal": cfg.causal,
                   "l2": "flushed between timed steps (256 MB write, outside the events)"},
        "block_tflops": flops / (ours_ms / 1e3) / 1e12,
        "gpu_launches": 7 * args.steps,
        "all_true_mask": {"ms_per_step": masked_ms, "value": T / (masked_ms / 1e3),
                          "equal_to_no_mask": bool(torch.equal(out, out_m))},
        "torch_eager": {"ms_per_step": torch_ms, "value": T / (torch_ms / 1e3),
                        "max_abs_diff_vs_ours": err},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def run_shape(args):
    """One of the reference's 14 official whole-model shapes (Project/shapes.json)
    through the drop-in model, timed as the reference benchmark times it (the
    same input every call, an all-true valid_token_mask, CUDA events around
    each forward; Ref :477-508): the default path (CUDA-graph replay from the
    second call for launch-bound sizes), the same model eagerly, and the
    PyTorch model of the oracle (BaselineTransformer restated, dense attention)
    on the same GPU for context."""
    import types
    from oracle import generate_case
    from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef
    from tiktok_techjam_2026_track3_b200 import ops, plugin
    from tiktok_techjam_2026_track3_b200.config import OFFICIAL_SHAPES
    sh = OFFICIAL_SHAPES[args.shape]
    dev = torch.device("cuda", 0)
    dtype = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[args.dtype]
    B = args.batch or sh.batch
    cfg = TransformerConfigRef(batch_size=B, seq_len=sh.seq_len, d_model=sh.d_model, num_heads=sh.num_heads,
                               ffn_dim=sh.ffn_dim, num_layers=sh.num_layers, causal=sh.causal)
    torch.manual_seed(1234)
    ref = BaselineTransformerRef(cfg)
    otb = types.SimpleNamespace(BaselineTransformer=BaselineTransformerRef)
    ours = plugin.build(otb, cfg)
    ours.load_state_dict(ref.state_dict())
    ours = ours.to(device=dev, dtype=dtype).eval()
    ref = ref.to(device=dev, dtype=dtype).eval()
    x, mask = generate_case(B, sh.seq_len, sh.d_model, 1234, dtype=dtype, device="cuda")
    stream = torch.cuda.current_stream(dev)

    def time_model(fn):
        with torch.inference_mode():
            for _ in range(max(args.warmup, 3)):
                fn()
            torch.cuda.synchronize(dev)
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
            for a, b in evs:
                a.record(stream)
                fn()
                b.record(stream)
            torch.cuda.synchronize(dev)
        return statistics.median(a.elapsed_time(b) for a, b in evs)

    with ClockSampler(dev) as clk:
        graph_ms = time_model(lambda: ours(x, mask))
    ours.ttj_cuda_graphs = False
    eager_ms = time_model(lambda: ours(x, mask))
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True  # the reference script's CUDA setting (Ref :687-688)
    try:
        torch_ms = time_model(lambda: ref(x, mask))
    except torch.cuda.OutOfMemoryError:
        torch_ms = None
    torch.backends.cuda.matmul.allow_tf32 = old_tf32
    ops.check_device_status(dev)
    T = B * sh.seq_len
    D, F, L = sh.d_model, sh.ffn_dim, sh.num_layers
    flops = L * (2.0 * T * D * 4 * D + 2.0 * 2 * T * D * F
                 + 4.0 * B * sh.num_heads * sh.seq_len ** 2 * (D // sh.num_heads) * (0.5 if sh.causal else 1.0))
    launches = L * 7 + 1 + (2 if dtype == torch.float32 else 0)
    line = {
        "metric": f"whole-model forward tokens/s, official shape {args.shape}", "value": T / (graph_ms / 1e3),
        "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": graph_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic (seeded; x ~ N(0,1); nn.Linear / nn.LayerNorm default init, seeded)",
        "config": {"workload": f"shape{args.shape}_b{B}_s{sh.seq_len}_d{D}_h{sh.num_heads}_l{L}_f{F}_causal",
                   "same_input_every_call": True, "valid_token_mask": "all true"},
        "model_tflops": flops / (graph_ms / 1e3) / 1e12,
        "eager": {"ms_per_step": eager_ms, "value": T / (eager_ms / 1e3)},
        "torch_reference_model_same_gpu": (None if torch_ms is None else
                                           {"ms_per_step": torch_ms, "value": T / (torch_ms / 1e3),
                                            "note": "dense PyTorch BaselineTransformer, TF32 allowed as Ref :687-688"}),
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def run_shape14(args):
    """Official shape 14 (B32 S100000 D1024 H16, 2 layers, ffn 1024, causal;
    the dense reference model cannot run it: its score table alone is 640 GB
    per batch row) through the drop-in model, timed two ways:

    * ``value``: the reference's own long-context timing
      (Project/tools/shape14_eval.py:520-560): 32 serial B=1 slices, each
      freshly generated from the CUDA generator (seed ``(1234 + 100000) * 1000
      + batch_index``) outside the timed region, CUDA events around each
      forward, a repeat's time = the sum of its 32 slice times, median over
      repeats (at least 3, after 3 warm-up slices);
    * ``full_batch``: the 32 rows as one B=32 forward, inputs resident.

    The reference's published figure for the same workload (RTX 3060 Ti,
    Project/BOARD.md:39) rides along as context, not as a ratio."""
    import types
    from oracle import generate_case
    from oracle.block_ref import BaselineTransformerRef, TransformerConfigRef
    from tiktok_techjam_2026_track3_b200 import ops, plugin
    from tiktok_techjam_2026_track3_b200.config import OFFICIAL_SHAPES
    sh = OFFICIAL_SHAPES[14]
    dev = torch.device("cuda", 0)
    dtype = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[args.dtype]
    B = args.batch or sh.batch
    cfg = TransformerConfigRef(batch_size=B, seq_len=sh.seq_len, d_model=sh.d_model, num_heads=sh.num_heads,
                               ffn_dim=sh.ffn_dim, num_layers=sh.num_layers, causal=sh.causal)
    torch.manual_seed(1234)
    template = BaselineTransformerRef(cfg)
    ours = plugin.build(types.SimpleNamespace(BaselineTransformer=BaselineTransformerRef), cfg)
    ours.load_state_dict(template.state_dict(), strict=True)
    ours = ours.to(device=dev, dtype=dtype).eval()
    del template
    stream = torch.cuda.current_stream(dev)
    repeats = max(3, min(args.steps, 3))
    timing_seed = 1234 + 100000

    def fresh(b):
        return generate_case(1, sh.seq_len, sh.d_model, timing_seed * 1000 + b, dtype=dtype, device="cuda")

    with torch.inference_mode(), ClockSampler(dev) as clk:
        for w in range(max(3, args.warmup)):  # warm-up: single B=1 calls, never the full batch
            x, mask = fresh(w % B)
            ours(x, mask)
        torch.cuda.synchronize(dev)
        sums = []
        for _ in range(repeats):
            slice_ms = []
            for b in range(B):
                x, mask = fresh(b)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                out = ours(x, mask)
                e1.record(stream)
                e1.synchronize()
                slice_ms.append(e0.elapsed_time(e1))
                del out, x, mask
            sums.append(sum(slice_ms))
        slices_clocks = clk.summary()
    ops.check_device_status(dev)
    slices_ms = statistics.median(sums)
    torch.cuda.empty_cache()
    with torch.inference_mode():
        xs = torch.cat([fresh(b)[0] for b in range(B)])
        full = []
        ours(xs, None)  # warm-up at the full batch (weights already packed)
        torch.cuda.synchronize(dev)
        for _ in range(repeats):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            out = ours(xs, None)
            e1.record(stream)
            e1.synchronize()
            full.append(e0.elapsed_time(e1))
            del out
    ops.check_device_status(dev)
    full_ms = statistics.median(full)
    T = B * sh.seq_len
    D, F, L = sh.d_model, sh.ffn_dim, sh.num_layers
    flops = L * (2.0 * T * D * 4 * D + 2.0 * 2 * T * D * F
                 + 4.0 * B * sh.num_heads * sh.seq_len ** 2 * (D // sh.num_heads) * 0.5)
    launches = L * 7 + 1 + (2 if dtype == torch.float32 else 0)
    peaks = measured_peaks()
    line = {
        "metric": "whole-model forward tokens/s, official shape 14", "value": T / (slices_ms / 1e3),
        "unit": UNIT, "n_gpus": 1, "steps": repeats, "warmup": max(3, args.warmup), "ms_per_step": slices_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic (seeded B=1 slices from the CUDA generator; x ~ N(0,1); nn.Linear / nn.LayerNorm "
                "default init, seeded)",
        "config": {"workload": f"shape14_b{B}_s{sh.seq_len}_d{D}_h{sh.num_heads}_l{L}_f{F}_causal",
                   "timing": f"{B} serial B=1 slices per step (the reference's shape-14 evaluation)",
                   "l2": "inputs of 400 MB per slice (larger than L2)", "valid_token_mask": "all true"},
        "model_tflops": flops / (slices_ms / 1e3) / 1e12,
        "frac_of_bf16_peak": flops / (slices_ms / 1e3) / 1e12 / peaks["bf16_tflops"],
        "full_batch": {"ms_per_step": full_ms, "value": T / (full_ms / 1e3),
                       "model_tflops": flops / (full_ms / 1e3) / 1e12},
        "reference_published_context": {"ms_per_step": 48271.04, "hardware": "RTX 3060 Ti (sm_86)",
                                        "source": "Project/BOARD.md:39 (32 serial B=1 calls)"},
        "gpu_launches": launches * B * repeats,
        "clocks": slices_clocks,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.shape == 14:
        return run_shape14(args)
    if args.shape is not None:
        return run_shape(args)
    from tiktok_techjam_2026_track3_b200.config import PRESETS
    cfg = PRESETS[args.config]
    if args.batch:
        cfg = cfg.with_(batch=args.batch)
    if args.seq:
        cfg = cfg.with_(seq_len=args.seq)
    if args.batch or args.seq:  # the workload name says what actually ran
        cfg = cfg.with_(name=f"{PRESETS[args.config].name} (overridden: batch {cfg.batch}, seq_len {cfg.seq_len})")
    if args.impl == "reference":
        return run_reference(args, cfg)
    if args.block:
        return run_block(args, cfg)
    return run_ours(args, cfg)


if __name__ == "__main__":
    raise SystemExit(main())
