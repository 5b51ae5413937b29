"""Host-resident batches through a device module with the PCIe copies hidden.

A serving loop whose activations live in host memory pays a host-to-device
copy of every input and a device-to-host copy of every output; at benchmark
config 2 (32 MiB each way per batch) those copies take longer than the three
layer kernels.  ``HostPipeline`` overlaps them across batches: while batch i
runs on the compute stream, batch i+1 is copied in on a second stream and
batch i-1 copied out on a third (the two copy directions use separate copy
engines), with two device buffers per direction.  In steady state a batch
costs max(copy in, kernels, copy out) instead of their sum.

Every batch is still copied in from, and its result copied back to, pinned host
memory; only the order of independent work changes, so results equal calling
the module on each batch in turn (tests/test_gpu_pipeline.py).
"""

from __future__ import annotations

import contextlib
import os
from typing import Callable, Iterator, List, Optional, Sequence

import torch

__all__ = ["HostPipeline", "device_local_cpus", "near_device"]


def _parse_cpulist(text: str) -> List[int]:
    cpus: List[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.extend(range(int(a), int(b) + 1))
        else:
            cpus.append(int(part))
    return cpus


def device_local_cpus(device: torch.device) -> Optional[List[int]]:
    """CPUs close to the GPU (NVML's ideal CPU affinity of the device, read only;
    else the sysfs NUMA node of its PCI slot), or None if unknown."""
    props = torch.cuda.get_device_properties(device)
    try:
        import pynvml
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{props.uuid}")
        words = pynvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        cpus = [64 * w + b for w, mask in enumerate(words) for b in range(64) if (mask >> b) & 1]
        if cpus:
            return cpus
    except Exception:
        pass
    try:
        addr = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{addr}/numa_node") as f:
            node = int(f.read().strip())
        if node >= 0:
            with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
                return _parse_cpulist(f.read())
    except (AttributeError, OSError, ValueError):
        pass
    return None


@contextlib.contextmanager
def near_device(device: torch.device) -> Iterator[Optional[List[int]]]:
    """Run the body with this process's CPU affinity restricted to the CPUs
    close to the GPU (``device_local_cpus``), then restore it.  Pinned host
    buffers allocated inside get their pages from memory local to those CPUs
    (first touch), so their PCIe copies do not cross the socket interconnect.
    Yields the CPU list (None when it cannot be determined; nothing changes)."""
    cpus = device_local_cpus(device)
    old = None
    if cpus and hasattr(os, "sched_setaffinity"):
        try:
            old = os.sched_getaffinity(0)
            os.sched_setaffinity(0, cpus)
        except OSError:
            old, cpus = None, None
    try:
        yield cpus
    finally:
        if old is not None:
            os.sched_setaffinity(0, old)


class HostPipeline:
    """Run ``fn`` (device tensor -> device tensor) over pinned host batches.

    ``depth`` device buffers per direction (2 overlaps one batch in flight on
    each side of the kernels).  ``fn`` is called under the compute stream, so
    modules from this package launch their kernels there.
    """

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor], device: torch.device,
                 depth: int = 2) -> None:
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.fn = fn
        self.device = torch.device(device)
        self.depth = depth
        self.h2d = torch.cuda.Stream(self.device)
        self.comp = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self._in: List[torch.Tensor] = []

    def _buffers(self, like: torch.Tensor) -> None:
        if (not self._in or self._in[0].shape != like.shape or self._in[0].dtype != like.dtype):
            self._in = [torch.empty(like.shape, dtype=like.dtype, device=self.device)
                        for _ in range(self.depth)]

    def run(self, host_inputs: Sequence[torch.Tensor], host_outputs: Sequence[torch.Tensor]) -> None:
        """Compute ``host_outputs[i] = fn(host_inputs[i])`` for every i.  Host
        tensors should be pinned (otherwise the copies are not asynchronous).
        Returns once the work is queued; the caller synchronises (or records an
        event on ``self.d2h``) before reading ``host_outputs``."""
        if len(host_inputs) != len(host_outputs):
            raise ValueError("one output per input")
        if not host_inputs:
            return
        self._buffers(host_inputs[0])
        d = self.depth
        caller = torch.cuda.current_stream(self.device)
        for s in (self.h2d, self.comp, self.d2h):
            s.wait_stream(caller)  # start after whatever the caller queued
        in_ready = [torch.cuda.Event() for _ in range(d)]
        comp_done = [torch.cuda.Event() for _ in range(d)]
        out_read = [torch.cuda.Event() for _ in range(d)]
        for i, (xh, oh) in enumerate(zip(host_inputs, host_outputs)):
            k = i % d
            with torch.cuda.stream(self.h2d):
                if i >= d:
                    self.h2d.wait_event(comp_done[k])  # batch i-d no longer reads this buffer
                self._in[k].copy_(xh, non_blocking=True)
                in_ready[k].record(self.h2d)
            with torch.cuda.stream(self.comp):
                self.comp.wait_event(in_ready[k])
                if i >= d:
                    self.comp.wait_event(out_read[k])  # bounds the device memory in flight
                y = self.fn(self._in[k])
                comp_done[k].record(self.comp)
            y.record_stream(self.d2h)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(comp_done[k])
                oh.copy_(y, non_blocking=True)
                out_read[k].record(self.d2h)
        caller.wait_stream(self.d2h)
