"""Batch sharding over the GPUs of one box (one process per GPU).

Images are independent, so a global batch is split into contiguous slices,
one per rank, with no data-path exchange; the only collective is the final
all-gather of the int32 predictions (and, optionally, the last-layer
outputs).  With NCCL on B200s that gather runs over NVLink; the same code runs
on `gloo` for CPU tests.  Uneven slices are padded to the largest slice for the
collective and trimmed afterwards.
"""
from __future__ import annotations


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) of rank's slice; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather(local, total: int, world: int, group=None):
    """All-gather a per-rank tensor [n_local, ...] into [total, ...] in rank
    order (torch.distributed must be initialised)."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return local
    n_max = max(b - a for a, b in (shard_bounds(total, world, r) for r in range(world)))
    pad = torch.zeros((n_max,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    buf = torch.empty((world * n_max,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, pad, group=group)
    parts = []
    for r in range(world):
        a, b = shard_bounds(total, world, r)
        parts.append(buf[r * n_max: r * n_max + (b - a)])
    return torch.cat(parts, 0)


def run_sharded(infer_local, x_global, world: int, rank: int, group=None):
    """Run `infer_local(x_slice) -> (out, pred)` on this rank's slice of the
    global batch and gather every rank's outputs and predictions."""
    total = x_global.shape[0]
    a, b = shard_bounds(total, world, rank)
    out, pred = infer_local(x_global[a:b])
    return gather(out, total, world, group), gather(pred, total, world, group)
