"""Host-in / host-out serving loop with the copies overlapped.

The reference has no such entry point: its benchmark keeps inputs resident on
the GPU. A caller whose batches live in host memory pays a host->device copy
of x (and the mask) and a device->host copy of the output per batch, which
for the small layers here costs more than the layer itself. HostPipeline runs
a sequence of batches through a model with three CUDA streams:

    copy-in stream    x_host[i] -> x_dev[i % 2]            (pinned, async)
    compute stream    y[i] = model(x_dev[i % 2], m_dev[i % 2])
    copy-out stream   y[i] -> out_host[i]                  (pinned, async)

so batch i+1's copy-in and batch i-1's copy-out run while batch i computes
(PCIe is full duplex). Every batch's own copies still happen; only their
overlap with neighbouring batches' work is new. Device buffers (input,
mask, output) are double buffered and guarded by events: an input slot is
refilled only after the forward that read it has finished, and an output slot
is rewritten only after its copy-out has finished. With a model that has
forward_into (OptimizedTransformer) nothing is allocated per batch.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch


class HostPipeline:
    """Overlapped host->device, forward, device->host over many batches.

    model: a callable forward(x, valid_token_mask) on `device`.
    run() takes equal-shape pinned host batches and pinned output buffers and
    returns once every output is in host memory.
    """

    def __init__(self, model: Callable, device: torch.device,
                 before_compute: Optional[Callable[[], None]] = None) -> None:
        self.model = model
        # writes into the pipeline's own output slots when the model can
        self._into = getattr(model, "forward_into", None)
        self.device = torch.device(device)
        self.before_compute = before_compute
        self.copy_in = torch.cuda.Stream(self.device)
        self.compute = torch.cuda.Stream(self.device)
        self.copy_out = torch.cuda.Stream(self.device)
        self._x: List[Optional[torch.Tensor]] = [None, None]
        self._m: List[Optional[torch.Tensor]] = [None, None]
        self._y: List[Optional[torch.Tensor]] = [None, None]

    def _slot_buffers(self, slot: int, x: torch.Tensor, m: Optional[torch.Tensor]):
        xd = self._x[slot]
        if xd is None or xd.shape != x.shape or xd.dtype != x.dtype:
            xd = self._x[slot] = torch.empty(x.shape, dtype=x.dtype, device=self.device)
        md = None
        if m is not None:
            md = self._m[slot]
            if md is None or md.shape != m.shape or md.dtype != m.dtype:
                md = self._m[slot] = torch.empty(m.shape, dtype=m.dtype, device=self.device)
        yd = self._y[slot]
        if yd is None or yd.shape != x.shape or yd.dtype != x.dtype:
            yd = self._y[slot] = torch.empty(x.shape, dtype=x.dtype, device=self.device)
        return xd, md, yd

    def run(self, xs: Sequence[torch.Tensor], masks: Optional[Sequence[Optional[torch.Tensor]]],
            outs: Sequence[torch.Tensor], start_event: Optional[torch.cuda.Event] = None,
            end_event: Optional[torch.cuda.Event] = None) -> None:
        """outs[i] <- model(xs[i], masks[i]) for every i, all host tensors.

        start_event / end_event (optional) are recorded before the first
        copy-in and after the last copy-out, for device-side timing.
        """
        n = len(xs)
        if len(outs) != n or (masks is not None and len(masks) != n):
            raise ValueError("xs, masks and outs must have the same length")
        in_done = [torch.cuda.Event() for _ in range(2)]
        compute_done = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]
        have_compute = [False, False]
        if start_event is not None:
            start_event.record(self.copy_in)
        for i in range(n):
            slot = i & 1
            m_host = masks[i] if masks is not None else None
            xd, md, yd = self._slot_buffers(slot, xs[i], m_host)
            with torch.cuda.stream(self.copy_in):
                if have_compute[slot]:
                    # the forward two batches back has finished reading this slot
                    self.copy_in.wait_event(compute_done[slot])
                xd.copy_(xs[i], non_blocking=True)
                if md is not None:
                    md.copy_(m_host, non_blocking=True)
                in_done[slot].record(self.copy_in)
            with torch.cuda.stream(self.compute):
                self.compute.wait_event(in_done[slot])
                if have_compute[slot]:
                    # the copy-out two batches back has finished reading yd
                    self.compute.wait_event(out_done[slot])
                if self.before_compute is not None:
                    self.before_compute()
                if self._into is not None:
                    self._into(xd, md, yd)
                else:
                    yd.copy_(self.model(xd, md))
                compute_done[slot].record(self.compute)
                have_compute[slot] = True
            with torch.cuda.stream(self.copy_out):
                self.copy_out.wait_event(compute_done[slot])
                outs[i].copy_(yd, non_blocking=True)
                out_done[slot].record(self.copy_out)
        if end_event is not None:
            end_event.record(self.copy_out)
        self.copy_out.synchronize()
