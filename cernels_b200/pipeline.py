"""Host-to-host execution of an experts step with copies overlapped with compute.

For callers whose tokens live in host memory: the batch is split into token chunks; chunk
c+1 is copied host->device on one stream while chunk c runs on the compute stream and chunk
c-1 is copied device->host on a third stream. Tokens are independent in every MoE-experts
operator (routing, expert MLPs and the combine are per token), so the result equals running
the whole batch at once.
"""

from __future__ import annotations

from typing import Callable

import torch


class HostPipeline:
    """Reusable device buffers and streams for `run`."""

    def __init__(self, device=None):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.copy_in = torch.cuda.Stream(self.device)
        self.copy_out = torch.cuda.Stream(self.device)
        self._bufs: dict = {}

    def _buffer(self, key, like: torch.Tensor) -> torch.Tensor:
        b = self._bufs.get(key)
        if b is None or b.shape != like.shape or b.dtype != like.dtype:
            b = torch.empty(like.shape, dtype=like.dtype, device=self.device)
            self._bufs[key] = b
        return b

    @staticmethod
    def chunk_bounds(T: int, chunks: int, taper: bool = False) -> list[int]:
        """Token boundaries of the chunks. With taper, the first and last chunks are half the size
        of the others, so the pipeline fills (first copy in) and drains (last copy out) faster."""
        chunks = max(1, min(int(chunks), T))
        if not taper or chunks < 3:
            return [(T * c) // chunks for c in range(chunks + 1)]
        units = 2 * chunks - 2  # half-size first and last chunks, full-size (2 units) middle ones
        edges = [0, 1] + [1 + 2 * c for c in range(1, chunks - 1)] + [units]
        bounds = [(T * e) // units for e in edges]
        if any(b <= a for a, b in zip(bounds[:-1], bounds[1:])):  # too few tokens: equal chunks
            return [(T * c) // chunks for c in range(chunks + 1)]
        return bounds

    def run(self, step: Callable, host_inputs: list[torch.Tensor], out_host: torch.Tensor, chunks: int = 4,
            taper: bool = False):
        """step(*device_chunks) -> device output rows for those tokens. host_inputs are pinned
        [T, ...] tensors split along dim 0; out_host is a pinned [T, ...] tensor, written."""
        T = host_inputs[0].shape[0]
        bounds = self.chunk_bounds(T, chunks, taper)
        chunks = len(bounds) - 1
        dev_in = [self._buffer(("in", i), t) for i, t in enumerate(host_inputs)]
        compute = torch.cuda.current_stream(self.device)
        self.copy_in.wait_stream(compute)   # buffers are free once earlier work finished
        self.copy_out.wait_stream(compute)
        ready = []
        for c in range(chunks):
            a, b = bounds[c], bounds[c + 1]
            with torch.cuda.stream(self.copy_in):
                for d, h in zip(dev_in, host_inputs):
                    d[a:b].copy_(h[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.copy_in)
            ready.append(ev)
        for c in range(chunks):
            a, b = bounds[c], bounds[c + 1]
            compute.wait_event(ready[c])
            y = step(*[d[a:b] for d in dev_in])
            done = torch.cuda.Event()
            done.record(compute)
            with torch.cuda.stream(self.copy_out):
                self.copy_out.wait_event(done)
                y.record_stream(self.copy_out)
                out_host[a:b].copy_(y, non_blocking=True)
        compute.wait_stream(self.copy_out)
        return out_host
