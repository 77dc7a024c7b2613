"""Inference over batches that live in host memory, with the host-to-device
copy of each batch overlapped with the forward of the previous one.

The reference runs one batch at a time: ``input_tensor.cuda()`` then
``model(input)`` (vit_cuda/model.py:185-199), so the copy and the forward are
serialised. ``StreamedInference`` keeps two device input buffers: batch i is
copied on a dedicated copy stream into the buffer the forward of batch i-2 has
finished with, and the forward of batch i (on the caller's current stream)
waits for that copy only. Each batch's logits are copied back on the current
stream into a pinned host tensor.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch


class StreamedInference:
    """``run = StreamedInference(model, (B, 3, H, W)); out = run(x_pinned)``
    enqueues one batch and returns the pinned host tensor its logits will land
    in (valid once the current stream is synchronised). ``fn`` replaces the
    forward (default ``model``), e.g. to all-gather logits across ranks.

    The call returns before the batch has left host memory: the copy from
    ``x_host`` runs asynchronously on the copy stream. ``x_host`` must not be
    modified until that copy is done — wait on ``input_copied()`` (or for the
    logits, which come later) before refilling the same host buffer."""

    def __init__(self, model, batch_shape, fn: Optional[Callable] = None):
        self.model = model
        self.fn = fn if fn is not None else model
        self.device = model.patch_weight.device
        self.copy_stream = torch.cuda.Stream(self.device)
        self.bufs = [torch.empty(batch_shape, dtype=torch.float32, device=self.device)
                     for _ in range(2)]
        self.copied = [torch.cuda.Event() for _ in range(2)]
        self.consumed = [torch.cuda.Event() for _ in range(2)]
        self.i = 0
        self.last = None

    def input_copied(self) -> Optional[torch.cuda.Event]:
        """The event recorded after the latest call's host-to-device copy: once
        it has completed (``.synchronize()`` / ``.query()``), that call's host
        input may be overwritten. None before the first call."""
        return None if self.last is None else self.copied[self.last]

    def __call__(self, x_host: torch.Tensor, out_host: Optional[torch.Tensor] = None):
        if x_host.device.type != "cpu":
            raise RuntimeError("StreamedInference: x_host must be a host tensor (pinned for overlap)")
        k = self.i % 2
        self.i += 1
        buf = self.bufs[k]
        if tuple(x_host.shape) != tuple(buf.shape):
            raise RuntimeError(f"StreamedInference: expected a batch of shape {tuple(buf.shape)}")
        compute = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(self.consumed[k])  # the forward two batches ago is done
            buf.copy_(x_host, non_blocking=True)
            self.copied[k].record(self.copy_stream)
        compute.wait_event(self.copied[k])
        with torch.no_grad():
            logits = self.fn(buf)
        self.consumed[k].record(compute)
        self.last = k
        if out_host is None:
            out_host = torch.empty(tuple(logits.shape), dtype=logits.dtype, pin_memory=True)
        out_host.copy_(logits, non_blocking=True)
        return out_host
