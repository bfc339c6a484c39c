"""Data-parallel replicas: one full model per GPU, the image batch split across ranks.

The W4A4 ViT forward has no exchange step between images, so the multi-GPU path is N independent
replicas (one process per GPU, ``torch.distributed`` over NCCL for the plumbing) with exactly two
collectives per measurement, both outside the per-image hot path: a MAX all-reduce of the device
timings and one all-gather of the logits at the end.  The same functions run on CPU ranks with
the gloo backend, which is how their logic and failure behaviour are tested.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def shard_range(global_batch: int, rank: int, world: int) -> tuple[int, int]:
    """(start, count) of ``rank``'s images: an even split, the first ``global_batch % world``
    ranks taking one extra image."""
    if world <= 0 or not 0 <= rank < world or global_batch < 0:
        raise ValueError(f"bad shard request: batch={global_batch} rank={rank} world={world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def init_from_env(backend: str, timeout_s: float = 120.0, device: torch.device | None = None):
    """Initialise the default process group from RANK / WORLD_SIZE / MASTER_* (127.0.0.1 default)."""
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kw = {}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist.get_rank(), dist.get_world_size()


def max_over_ranks(values: list[float], device: torch.device | str = "cpu") -> list[float]:
    """Element-wise MAX of per-rank measurements (identity when not distributed)."""
    t = torch.tensor(values, dtype=torch.float64 if str(device) == "cpu" else torch.float32, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def gather_logits(local: torch.Tensor, global_batch: int) -> torch.Tensor | None:
    """All-gather every rank's (count_r, C) logits into the (global_batch, C) batch order.

    Uneven shards are padded to the largest shard for the collective and trimmed after.
    Returns the full tensor on every rank (None is never returned when distributed)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    world = dist.get_world_size()
    counts = [shard_range(global_batch, r, world)[1] for r in range(world)]
    cmax = max(counts)
    pad = local.new_zeros((cmax, *local.shape[1:]))
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous())
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
