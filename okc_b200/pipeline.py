"""Double-buffered host I/O around a device step, for serving throughput.

A step whose input comes from host memory and whose result goes back to it pays two PCIe
copies on top of its device time when they run in series with it (the C4 decode layer: 2 MB
in and 2 MB out, ~40 us each, around a ~330 us step).  HostPipeline overlaps them.  Step k's
input copy (host -> device) and step k-1's output copy (device -> host) run on the copy
engines, each on its own stream.  Meanwhile step k computes on a third stream, where the step
is replayed as a CUDA graph.  Two device input buffers and two output buffers alternate, and
events order every reuse:

    copy-in  k  into in[i]    after compute k-2 has finished reading in[i]
    compute  k  from in[i]    after copy-in k, and after copy-out k-2 has finished reading out[i]
    copy-out k  from out[i]   after compute k

Every submitted step has its input copied in and its result copied out.  Steps run on the
device in submission order on one stream, so a stateful step (a KV-cache append) sees the same
state as it would in series.  Host buffers must be pinned.  A host output buffer is written
asynchronously: read it after synchronize(), or after the step's copy-out has completed.
"""

from __future__ import annotations

from typing import Callable

import torch


class HostPipeline:
    """step(inp) -> out: `inp` is a uint8 device tensor of in_nbytes (the step views it as its
    inputs); `out` is the device tensor to copy back.  The step is captured into one CUDA graph
    per input buffer.  It must allocate its output inside the call (the graph keeps that memory
    as its static output, one per buffer) or return a view of it, and must accept an all-zero
    input (it runs once per buffer on zeros before capture, for lazy initialisation)."""

    def __init__(self, step: Callable[[torch.Tensor], torch.Tensor], in_nbytes: int, device):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("HostPipeline runs CUDA steps only")
        self.s_in = torch.cuda.Stream(self.device)
        self.s_run = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self.inp = [torch.zeros(in_nbytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self.graphs: list[torch.cuda.CUDAGraph] = []
        self.out: list[torch.Tensor] = []
        cur = torch.cuda.current_stream(self.device)
        for i in range(2):
            self.s_run.wait_stream(cur)
            with torch.cuda.stream(self.s_run):
                step(self.inp[i])
            cur.wait_stream(self.s_run)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                o = step(self.inp[i])
            self.graphs.append(g)
            self.out.append(o)
        if self.out[0].data_ptr() == self.out[1].data_ptr():
            raise RuntimeError("the step must allocate its output per call (both graphs write one buffer)")
        torch.cuda.synchronize(self.device)
        self.ev_in = [torch.cuda.Event() for _ in range(2)]
        self.ev_run = [torch.cuda.Event() for _ in range(2)]
        self.ev_out = [torch.cuda.Event() for _ in range(2)]
        self.k = 0
        self._checked: set = set()

    def submit(self, host_in: torch.Tensor, host_out: torch.Tensor) -> None:
        """Enqueues one step: host_in (pinned, in_nbytes) in, the step, its output into host_out
        (pinned, the output's shape and dtype).  Returns without waiting."""
        i = self.k & 1
        key = (host_in.data_ptr(), host_in.numel(), host_out.data_ptr(), tuple(host_out.shape), host_out.dtype)
        if key not in self._checked:  # checked once per buffer pair (is_pinned asks the driver)
            if not (host_in.is_pinned() and host_out.is_pinned()):
                raise RuntimeError("HostPipeline needs pinned host buffers (unpinned copies would not overlap)")
            if host_in.numel() * host_in.element_size() != self.inp[i].numel():
                raise RuntimeError("host_in must hold exactly the step's input bytes")
            if host_out.shape != self.out[i].shape or host_out.dtype != self.out[i].dtype:
                raise RuntimeError(f"host_out must be {tuple(self.out[i].shape)} {self.out[i].dtype}")
            self._checked.add(key)
        self.s_in.wait_event(self.ev_run[i])
        with torch.cuda.stream(self.s_in):
            self.inp[i].copy_(host_in, non_blocking=True)
        self.ev_in[i].record(self.s_in)
        self.s_run.wait_event(self.ev_in[i])
        self.s_run.wait_event(self.ev_out[i])
        with torch.cuda.stream(self.s_run):
            self.graphs[i].replay()
        self.ev_run[i].record(self.s_run)
        self.s_out.wait_event(self.ev_run[i])
        with torch.cuda.stream(self.s_out):
            host_out.copy_(self.out[i], non_blocking=True)
        self.ev_out[i].record(self.s_out)
        self.k += 1

    def synchronize(self) -> None:
        for s in (self.s_in, self.s_run, self.s_out):
            s.synchronize()

    def close(self) -> None:
        """Releases the graphs (graphs that hold NCCL calls must go before the process group)."""
        self.synchronize()
        self.graphs.clear()
        self.out.clear()
