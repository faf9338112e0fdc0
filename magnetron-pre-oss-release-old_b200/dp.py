"""Row-sharded data parallelism for the multi-GPU paths.

The MLP batch (and any row-independent workload) is split by rows over one
process per GPU; every rank runs the same program on its rows and the outputs
are collected with one all-gather.  These helpers are backend-agnostic:
`torch.distributed` with NCCL on B200s (the collective runs on the device's
stream), gloo on CPU in the tests.
"""
from __future__ import annotations


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s shard; shards differ by at most one row."""
    base, rem = divmod(total, world)
    rows = base + (1 if rank < rem else 0)
    start = rank * base + min(rank, rem)
    return start, rows


def gather_rows(local, total_rows: int, row_width: int, world: int, rank: int):
    """All-gather row shards (each rank's `local` holds its rows x row_width values,
    flattened) into the full total_rows x row_width buffer, in rank order."""
    import torch
    import torch.distributed as dist

    if total_rows % world == 0:  # equal shards: gather straight into the result
        out = torch.empty(total_rows * row_width, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.reshape(-1)[: (total_rows // world) * row_width])
        return out
    cap = (total_rows + world - 1) // world
    padded = torch.zeros(cap * row_width, dtype=local.dtype, device=local.device)
    _, rows = shard_rows(total_rows, world, rank)
    padded[: rows * row_width] = local.reshape(-1)[: rows * row_width]
    out = torch.empty(world * cap * row_width, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, padded)
    parts = []
    for r in range(world):
        _, n = shard_rows(total_rows, world, r)
        parts.append(out[r * cap * row_width: r * cap * row_width + n * row_width])
    return torch.cat(parts)


def gather_records(local, world: int):
    """All-gather one fixed-size record per rank (a 1-D tensor, same length on every
    rank) into world records in rank order."""
    import torch
    import torch.distributed as dist

    out = torch.empty(world * local.numel(), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local)
    return out


def reduce_full(dev, name: str, shard, r_ptr: int, world: int):
    """Full SUM/MEAN/MIN/MAX of a tensor whose elements are split over the ranks
    (`shard` is this rank's part, a backend tensor): one record per rank (double
    sum, min, max, count), an all-gather of the world records in rank order on
    the backend's stream, and a fixed-order combine into r[0] on every rank.
    The exchange is 24 bytes per rank."""
    import torch

    device = torch.device("cuda", dev.ordinal)
    stream = torch.cuda.ExternalStream(dev.stream, device=device)
    with torch.cuda.stream(stream):
        mine = torch.empty(3, dtype=torch.float64, device=device)  # one 24-byte record, 8-byte aligned
        dev.reduce_partial(shard, mine.data_ptr())
        parts = gather_records(mine, world)
        dev.reduce_combine(name, r_ptr, parts.data_ptr(), world)
        mine.record_stream(stream)
        parts.record_stream(stream)
