"""Host-to-host serving loop with copy/compute overlap.

A serving step takes a batch of hidden states from host memory, runs the layer
and returns the result to host memory.  Run back to back on one stream, the two
PCIe/C2C copies serialise with the layer (the prefill batch is 128 MiB each
way).  :class:`HostPipeline` keeps ``depth`` device input buffers and moves the
copies to their own stream:

* the host->device copy of batch i+1 runs while batch i computes;
* the device->host copy of batch i's output runs while batch i+1 computes;
* the two directions have a stream each, so they overlap one another too (a
  link carries both directions at once; on one stream they would add up).

Every batch's copies still happen (and are waited for at the end of
:meth:`HostPipeline.run`); only their overlap with compute changes.  The
layer callable runs on the caller's current stream, unchanged.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch


class HostPipeline:
    """``fn(device_batch) -> device_out`` (or a tuple whose first item is the
    output) over host batches, with double-buffered (``depth``) inputs.

    ``run(inputs, outputs)`` takes pinned host tensors: ``inputs[i]`` is copied
    to the device, ``fn`` is applied, and its output is copied into
    ``outputs[i]``.  Returns after every output has landed in host memory.
    """

    def __init__(self, fn: Callable, like: torch.Tensor, device: torch.device, depth: int = 2):
        self.fn = fn
        self.depth = max(1, int(depth))
        self.device = device
        self.bufs = [torch.empty(like.shape, dtype=like.dtype, device=device)
                     for _ in range(self.depth)]
        self.copy_stream = torch.cuda.Stream(device=device)      # host -> device
        self.out_stream = torch.cuda.Stream(device=device)       # device -> host
        # buffer b may be overwritten once the compute that read it finished
        self._free = [None] * self.depth
        # outputs whose device->host copy may still run, with that copy's event:
        # held (instead of record_stream, whose deferred frees make every later
        # allocation poll events) until the compute stream has waited for it
        self._held = [None] * self.depth

    def run(self, inputs: Sequence[torch.Tensor], outputs: Sequence[torch.Tensor]) -> None:
        compute = torch.cuda.current_stream(self.device)
        cs, os_ = self.copy_stream, self.out_stream
        cs.wait_stream(compute)  # nothing of this run starts before the caller's prior work
        os_.wait_stream(compute)
        loaded = [None] * self.depth

        def load(i: int) -> None:
            b = i % self.depth
            with torch.cuda.stream(cs):
                if self._free[b] is not None:
                    cs.wait_event(self._free[b])
                self.bufs[b].copy_(inputs[i], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                loaded[b] = ev

        n = len(inputs)
        if n == 0:
            return
        load(0)
        for i in range(n):
            b = i % self.depth
            if i + 1 < n and self.depth > 1:
                load(i + 1)  # overlaps this batch's compute
            compute.wait_event(loaded[b])
            res = self.fn(self.bufs[b])
            out = res[0] if isinstance(res, (tuple, list)) else res
            done = torch.cuda.Event()
            done.record(compute)
            self._free[b] = done
            if self._held[b] is not None:
                # the copy of the output `depth` steps ago is ordered before any
                # later use of its memory on the compute stream
                compute.wait_event(self._held[b][1])
            with torch.cuda.stream(os_):
                os_.wait_event(done)
                outputs[i].copy_(out, non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(os_)
            self._held[b] = (out, copied)
            if self.depth == 1 and i + 1 < n:
                load(i + 1)
        cs.synchronize()
        os_.synchronize()
        compute.wait_stream(cs)
        compute.wait_stream(os_)
        self._held = [None] * self.depth
