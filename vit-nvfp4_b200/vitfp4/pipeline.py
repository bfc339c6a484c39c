"""Host-fed inference with the transfers overlapped: batch i+1's host -> device copy and batch i-1's
device -> host read of the logits run on a copy stream while batch i's forward runs.

Every batch still crosses PCIe / C2C in both directions; only their order against the forward
changes.  Two device input buffers alternate: the copy of batch i+2 into a buffer waits for the
forward of batch i, the last reader of that buffer, and the read-back of batch i waits for its
forward.  ``run`` returns when every read-back has landed in the pinned host outputs.
"""
from __future__ import annotations

import torch


class OverlappedRunner:
    """``model`` over pinned host batches, copies on a second CUDA stream.

    model(x) -> logits on ``device``; ``out_fn`` maps the logits to the tensor read back
    (default: fp32).  Host batches must be pinned (page-locked) for the copies to be
    asynchronous and must all have the same shape and dtype."""

    def __init__(self, model, device: torch.device, out_fn=None):
        self.model = model
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("OverlappedRunner needs a CUDA device")
        self.out_fn = out_fn if out_fn is not None else (lambda t: t.float())
        self.copy_stream = torch.cuda.Stream(self.device)
        self._bufs: list[torch.Tensor] = []

    def _buffers(self, like: torch.Tensor) -> list[torch.Tensor]:
        if not self._bufs or self._bufs[0].shape != like.shape or self._bufs[0].dtype != like.dtype:
            self._bufs = [torch.empty(like.shape, dtype=like.dtype, device=self.device) for _ in range(2)]
        return self._bufs

    def run(self, host_batches: list[torch.Tensor], host_outs: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
        """Forward every batch; returns the read-back outputs (pinned host tensors) in order.
        The work is ordered after everything already queued on the current stream, and the current
        stream waits for the last read-back, so events recorded around the call time all of it."""
        n = len(host_batches)
        if n == 0:
            return []
        for hb in host_batches:
            if hb.device.type != "cpu":
                raise ValueError("host_batches must be host tensors")
        compute = torch.cuda.current_stream(self.device)
        copy = self.copy_stream
        bufs = self._buffers(host_batches[0])
        copied = [torch.cuda.Event() for _ in range(n)]
        computed = [torch.cuda.Event() for _ in range(n)]
        outs: list[torch.Tensor | None] = [None] * n if host_outs is None else list(host_outs)
        copy.wait_stream(compute)                     # nothing starts before the caller's prior work

        def h2d(i: int):
            with torch.cuda.stream(copy):
                if i >= 2:
                    copy.wait_event(computed[i - 2])  # the forward of batch i-2 read this buffer
                bufs[i % 2].copy_(host_batches[i], non_blocking=True)
                copied[i].record(copy)

        h2d(0)
        for i in range(n):
            if i + 1 < n:
                h2d(i + 1)
            compute.wait_event(copied[i])
            y = self.out_fn(self.model(bufs[i % 2]))
            computed[i].record(compute)
            with torch.cuda.stream(copy):
                copy.wait_event(computed[i])
                if outs[i] is None:
                    outs[i] = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
                outs[i].copy_(y, non_blocking=True)
            y.record_stream(copy)                      # y stays allocated until its read-back ran
        compute.wait_stream(copy)
        return outs
