"""Batches held in pinned host memory through a block, copies overlapped with compute.

The reference's block benchmark (block_benchmark.py) times a block on tensors
already on the GPU; a serving loop around it copies each batch in, runs the
block and copies the result out, one after the other.  `HostPipeline` keeps
`slots` device buffers and two copy streams: while batch i computes on the
caller's stream, batch i+1's host→device copy and batch i-1's device→host copy
run on the copy engines, so once the pipe is full a step costs
max(compute, copies) instead of their sum.  Every batch is still copied in and
out in full; nothing is cached between batches.

With ``graphs=True`` each slot's forward is captured once as a CUDA graph
(after a warm-up on that slot's buffers) and replayed, so a step costs one
graph launch on the host instead of the block's per-kernel launches; the
block must be capturable (MoEBlock, or ExpertParallelMoEBlock on the p2p
backend).  The bits are those of the eager forward.

Dependencies, per slot s (events on the device, no host synchronisation):
    load(i)    waits computed[s] of batch i-slots (x[s] free), records loaded[s]
    compute(i) waits loaded[s] and stored[s] (y[s] free), records computed[s]
    store(i)   waits computed[s], records stored[s]

With one process per GPU on a multi-socket host, allocate each process's
pinned batches on the memory node of its GPU: `device_local_cpus(device)`
gives that GPU's local CPU set (from NVML), and pinned memory allocated while
the process runs on those CPUs is placed on their node.
"""

from __future__ import annotations

import os

import torch


def device_local_cpus(device):
    """The CPU cores attached to `device`'s socket, as a set (NVML's CPU
    affinity of the GPU, matched by PCI bus id), or None when NVML or the
    GPU's PCI location is not available.  Reads only; changes nothing."""
    try:
        import pynvml

        props = torch.cuda.get_device_properties(torch.device(device))
        bus_id = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus_id)
            words = (os.cpu_count() + 63) // 64
            mask = pynvml.nvmlDeviceGetCpuAffinity(handle, words)
        finally:
            pynvml.nvmlShutdown()
    except Exception:  # no NVML, no GPU, or a driver that does not report it
        return None
    cpus = {64 * w + b for w, bits in enumerate(mask) for b in range(64) if (int(bits) >> b) & 1}
    return cpus or None


def pinned_on_device_node(tensors, device):
    """Pinned copies of host `tensors`, allocated while this process runs on
    the CPUs local to `device` (so their pages land on that GPU's memory
    node); the process's CPU affinity is restored afterwards."""
    cpus = device_local_cpus(device)
    previous = os.sched_getaffinity(0) if hasattr(os, "sched_getaffinity") else None
    if cpus and previous is not None and cpus & previous:
        os.sched_setaffinity(0, cpus & previous)
    try:
        return [t.contiguous().pin_memory() for t in tensors]
    finally:
        if cpus and previous is not None:
            os.sched_setaffinity(0, previous)


class HostPipeline:
    """Run `block(x, out=y)` over pinned host batches of one shape.

    `block` is a `MoEBlock` or an `ExpertParallelMoEBlock` (anything whose
    forward accepts `out=`).  Host tensors must be pinned, contiguous and of the
    pipeline's shape and dtype; the caller must not touch them until `run`
    returns (or, with `synchronize=False`, until the caller's stream has
    passed the point where `run` returned).
    """

    def __init__(self, block, tokens, *, hidden=None, dtype=torch.bfloat16, device=None,
                 slots=2, graphs=False):
        if slots < 2:
            raise ValueError("a pipeline needs at least two slots")
        device = torch.device(device) if device is not None else block.gate_up_weight.device
        if device.type != "cuda":
            raise RuntimeError("HostPipeline drives a CUDA block")
        hidden = hidden or block.config.hidden
        self.block = block
        self.shape = (int(tokens), int(hidden))
        self.dtype = dtype
        self.device = device
        self.slots = slots
        self.x = [torch.zeros(self.shape, dtype=dtype, device=device) for _ in range(slots)]
        self.y = [torch.empty(self.shape, dtype=dtype, device=device) for _ in range(slots)]
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.loaded = [torch.cuda.Event() for _ in range(slots)]
        self.computed = [torch.cuda.Event() for _ in range(slots)]
        self.stored = [torch.cuda.Event() for _ in range(slots)]
        self.graphs = self._capture() if graphs else None

    @torch.inference_mode()
    def _capture(self):
        """One CUDA graph per slot of block(x[s], out=y[s]), captured on a side
        stream after a warm-up forward on the same buffers."""
        compute = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(compute)
        with torch.cuda.stream(side):
            for s in range(self.slots):
                self.block(self.x[s], out=self.y[s])
        compute.wait_stream(side)
        graphs = []
        for s in range(self.slots):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                self.block(self.x[s], out=self.y[s])
            graphs.append(graph)
        compute.wait_stream(side)
        torch.cuda.synchronize(self.device)
        return graphs

    def close(self):
        """Release the captured graphs (before the block's resources go)."""
        if self.graphs is not None:
            torch.cuda.synchronize(self.device)
            self.graphs = None

    def _check(self, tensors, what):
        for t in tensors:
            if t.device.type != "cpu" or not t.is_pinned():
                raise ValueError(f"{what} must be pinned host tensors")
            if tuple(t.shape) != self.shape or t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError(f"{what} must be contiguous {self.dtype} tensors of shape "
                                 f"{self.shape}")

    def bytes_per_batch(self):
        """(host→device, device→host) bytes copied for one batch."""
        n = self.shape[0] * self.shape[1] * torch.empty((), dtype=self.dtype).element_size()
        return n, n

    @torch.inference_mode()
    def run(self, inputs, outputs, synchronize=True):
        """outputs[i] = block(inputs[i]) for every i; returns `outputs`."""
        inputs, outputs = list(inputs), list(outputs)
        if len(inputs) != len(outputs):
            raise ValueError("inputs and outputs differ in length")
        self._check(inputs, "inputs")
        self._check(outputs, "outputs")
        compute = torch.cuda.current_stream(self.device)
        # copies start after whatever the caller queued before this call
        self.h2d.wait_stream(compute)
        self.d2h.wait_stream(compute)

        def load(i):
            s = i % self.slots
            self.h2d.wait_event(self.computed[s])
            with torch.cuda.stream(self.h2d):
                self.x[s].copy_(inputs[i], non_blocking=True)
            self.loaded[s].record(self.h2d)

        for i in range(min(self.slots - 1, len(inputs))):
            load(i)
        for i in range(len(inputs)):
            s = i % self.slots
            if i + self.slots - 1 < len(inputs):
                load(i + self.slots - 1)
            compute.wait_event(self.loaded[s])
            compute.wait_event(self.stored[s])
            if self.graphs is not None:
                self.graphs[s].replay()
            else:
                self.block(self.x[s], out=self.y[s])
            self.computed[s].record(compute)
            self.d2h.wait_event(self.computed[s])
            with torch.cuda.stream(self.d2h):
                outputs[i].copy_(self.y[s], non_blocking=True)
            self.stored[s].record(self.d2h)
        compute.wait_stream(self.h2d)
        compute.wait_stream(self.d2h)
        if synchronize:
            compute.synchronize()
        return outputs
