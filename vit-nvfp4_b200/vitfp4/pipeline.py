"""Serving helpers around a converted model: CUDA-graph replay of the forward, and host-fed inference
with the transfers overlapped.

``GraphedForward`` captures ``model(x)`` for one input shape as CUDA graphs and replays them: a W4A4
ViT-L/14 forward is ~400 kernel launches, and issuing them one by one through Python and ctypes costs
more host time than a small batch's device time, so replay is what keeps small per-GPU batches
device-bound.  The model must have run eagerly once on that shape first (calibration of static
globals, weight packing and similar one-time work happen there; nothing in the captured forward may
synchronise the host).

``OverlappedRunner`` runs batches from pinned host memory: batch i+1's host -> device copy and batch
i-1's device -> host read of the logits run on a copy stream while batch i's forward runs.  Every
batch still crosses PCIe / C2C in both directions; only their order against the forward changes.
"""
from __future__ import annotations

import torch


class GraphedForward:
    """``model`` captured as ``n_buffers`` CUDA graphs, one per static input buffer (all sharing one
    memory pool; they never run concurrently because they replay on one stream).

    ``forward(i)`` replays graph i on the current stream, reading ``inputs[i]`` and writing
    ``outputs[i]`` (both owned here and reused by every replay of graph i); ``__call__(x)`` copies x
    into buffer 0 and replays graph 0."""

    def __init__(self, model, example: torch.Tensor, n_buffers: int = 1, warmup: int = 1):
        if example.device.type != "cuda":
            raise RuntimeError("GraphedForward needs a CUDA input")
        self.model = model
        self.inputs = [torch.empty_like(example) for _ in range(n_buffers)]
        for b in self.inputs:
            b.copy_(example)
        side = torch.cuda.Stream(example.device)
        side.wait_stream(torch.cuda.current_stream(example.device))
        with torch.cuda.stream(side):           # eager warm-up off the capturing stream's history
            for _ in range(warmup):
                model(self.inputs[0])
        torch.cuda.current_stream(example.device).wait_stream(side)
        torch.cuda.synchronize(example.device)
        self.graphs, self.outputs = [], []
        pool = None
        for b in self.inputs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                out = model(b)
            pool = g.pool() if pool is None else pool
            self.graphs.append(g)
            self.outputs.append(out)

    def forward(self, i: int = 0) -> torch.Tensor:
        self.graphs[i].replay()
        return self.outputs[i]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        self.inputs[0].copy_(x, non_blocking=True)
        return self.forward(0)

    def release(self) -> None:
        """Free the graphs and their memory pool."""
        self.graphs, self.outputs, self.inputs = [], [], []


class OverlappedRunner:
    """``model`` over pinned host batches, copies on a second CUDA stream.

    model(x) -> logits on ``device``; ``out_fn`` maps the logits to the tensor read back
    (default: fp32).  Host batches must be pinned (page-locked) for the copies to be
    asynchronous and must all have the same shape and dtype.  With ``graphed`` the forward is
    replayed from two CUDA graphs (``GraphedForward``, one per device input buffer), captured on
    the first ``run``."""

    def __init__(self, model, device: torch.device, out_fn=None, graphed: bool = False):
        self.model = model
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("OverlappedRunner needs a CUDA device")
        self.out_fn = out_fn if out_fn is not None else (lambda t: t.float())
        self.copy_stream = torch.cuda.Stream(self.device)
        self.graphed = graphed
        self._bufs: list[torch.Tensor] = []
        self._graphs: GraphedForward | None = None

    def _buffers(self, like: torch.Tensor) -> list[torch.Tensor]:
        if not self._bufs or self._bufs[0].shape != like.shape or self._bufs[0].dtype != like.dtype:
            if self.graphed:
                example = like.to(self.device)
                fwd = lambda x: self.out_fn(self.model(x))   # noqa: E731  (the read-back tensor is a graph output)
                self._graphs = GraphedForward(fwd, example, n_buffers=2)
                self._bufs = self._graphs.inputs
            else:
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
        read = [torch.cuda.Event() for _ in range(n)]
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
            if self.graphed:
                if i >= 2:
                    compute.wait_event(read[i - 2])   # graph i % 2 rewrites the output read back at i-2
                y = self._graphs.forward(i % 2)
            else:
                y = self.out_fn(self.model(bufs[i % 2]))
            computed[i].record(compute)
            with torch.cuda.stream(copy):
                copy.wait_event(computed[i])
                if outs[i] is None:
                    outs[i] = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
                outs[i].copy_(y, non_blocking=True)
                read[i].record(copy)
            if not self.graphed:
                y.record_stream(copy)                  # y stays allocated until its read-back ran
        compute.wait_stream(copy)
        return outs
