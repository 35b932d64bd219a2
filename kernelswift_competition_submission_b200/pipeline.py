"""Batches that live in host memory, run through the MoE layer with the copies hidden.

A serving process usually holds its token batches in (pinned) host memory. Run
one after the other, every batch pays its host->device copy of the hidden
states and router logits, the layer, and the device->host copy of the result in
sequence. ``HostPipeline`` overlaps them on three CUDA streams with two device
buffers per input and output: while the layer works on batch i, the copy engine
brings batch i+1 in and takes batch i-1 out.

Ordering is kept by CUDA events only (the host waits once, for the last output):

    h2d  : waits layer(i-2) (buffer reuse)             -> copies batch i into slot i % 2
    layer: waits h2d(i), and d2h(i-2) (output reuse)   -> fn(x[slot], g[slot]) into out[slot]
    d2h  : waits layer(i)                              -> copies out[slot] to the host output

``fn`` is any callable on device tensors that launches on torch's current
stream (``moe_layer``, ``ExpertParallelMoE.forward``, ...). Results are the
same bits as calling ``fn`` batch by batch: the same kernels run on the same
inputs; only the copies move.
"""

from __future__ import annotations

import os
from pathlib import Path
from typing import Callable, Sequence

import torch


def parse_cpulist(text: str) -> set[int]:
    """CPU ids of a sysfs cpulist such as "0-23,96-119"."""
    cpus: set[int] = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-", 1)
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def gpu_local_cpus(device: torch.device | int, sysfs: str | Path = "/sys/bus/pci/devices") -> set[int]:
    """The host CPUs on the NUMA node the GPU hangs off (its PCI device's local_cpulist);
    an empty set when the platform does not say."""
    idx = device if isinstance(device, int) else (device.index or 0)
    p = torch.cuda.get_device_properties(idx)
    bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    f = Path(sysfs) / bdf / "local_cpulist"
    try:
        return parse_cpulist(f.read_text())
    except (OSError, ValueError):
        return set()


def bind_to_gpu_node(device: torch.device | int, sysfs: str | Path = "/sys/bus/pci/devices") -> set[int]:
    """Restrict this process to the CPUs local to the GPU (intersected with the ones it may
    use), so pinned host buffers allocated afterwards are placed on that NUMA node by first
    touch and host<->device copies do not cross the socket link. Returns the CPUs kept (the
    affinity is left alone when the intersection is empty)."""
    allowed = os.sched_getaffinity(0)
    local = gpu_local_cpus(device, sysfs) & allowed
    if local:
        os.sched_setaffinity(0, local)
    return local


class HostPipeline:
    def __init__(self, fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor], device: torch.device | int):
        self.fn = fn
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("HostPipeline runs on a CUDA device")
        self._slots = None
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)

    def _ensure(self, x: torch.Tensor, g: torch.Tensor):
        key = (tuple(x.shape), x.dtype, tuple(g.shape), g.dtype)
        if self._slots is not None and self._slots[0] == key:
            return self._slots[1]
        slots = [(torch.empty(x.shape, dtype=x.dtype, device=self.device),
                  torch.empty(g.shape, dtype=g.dtype, device=self.device)) for _ in range(2)]
        self._slots = (key, slots)
        return slots

    def run(self, xs: Sequence[torch.Tensor], gs: Sequence[torch.Tensor], outs: Sequence[torch.Tensor]) -> None:
        """Run fn over host batches ``xs[i], gs[i]`` into host ``outs[i]``; all tensors pinned,
        of one shape per argument. Returns when the last output has landed on the host."""
        n = len(xs)
        if not (len(gs) == n and len(outs) == n):
            raise ValueError("xs, gs and outs must have the same length")
        if n == 0:
            return
        for t in (*xs, *gs, *outs):
            if t.device.type != "cpu" or not t.is_pinned():
                raise ValueError("HostPipeline batches must be pinned host tensors")
        compute = torch.cuda.current_stream(self.device)
        slots = self._ensure(xs[0], gs[0])
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [None, None]   # the layer finished reading slot s
        out_free = [None, None]  # d2h finished reading the output of slot s
        with torch.cuda.device(self.device):
            # the copies start after the work queued before run() on the caller's stream
            self.h2d.wait_stream(compute)
            self.d2h.wait_stream(compute)

            def load(i):
                s = i % 2
                if in_free[s] is not None:
                    self.h2d.wait_event(in_free[s])
                with torch.cuda.stream(self.h2d):
                    slots[s][0].copy_(xs[i], non_blocking=True)
                    slots[s][1].copy_(gs[i], non_blocking=True)
                in_ready[s].record(self.h2d)

            load(0)
            for i in range(n):
                s = i % 2
                if i + 1 < n:  # issued before fn(i), which may block the host (e.g. on split sizes)
                    load(i + 1)
                compute.wait_event(in_ready[s])
                if out_free[s] is not None:
                    compute.wait_event(out_free[s])
                o = self.fn(*slots[s])
                done = torch.cuda.Event()
                done.record(compute)
                in_free[s] = done
                self.d2h.wait_event(done)
                o.record_stream(self.d2h)  # the allocator must not hand o's memory out before the copy ends
                with torch.cuda.stream(self.d2h):
                    outs[i].copy_(o, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.d2h)
                out_free[s] = ev
            compute.wait_stream(self.d2h)
        self.d2h.synchronize()
