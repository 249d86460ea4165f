"""Multi-GPU partitioning of the student-linear path (one process per GPU).

Every output row of a student linear depends only on its own token row, so a batch
shards by token rows with the weights replicated; a layer whose weight is too wide can
also shard its output columns.  No data-path collective is needed to compute the
shards; the collectives here are the optional gather of a full output and the global
Freivalds verdict (a sum of per-rank rejected-row counts).  They run on whatever backend
the process group has (NCCL on B200, gloo in the CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def row_shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous share of `total` rows (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def col_shard(total: int, world: int, rank: int, align: int = 16) -> tuple[int, int]:
    """[start, stop) of rank's share of `total` output columns, boundaries multiples of
    `align` (so each shard's rows stay 16-byte aligned for the GEMM's vector stores)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    units = (total + align - 1) // align
    s, e = row_shard(units, world, rank)
    return min(s * align, total), min(e * align, total)


def all_gather_rows(local: torch.Tensor, total_rows: int, group=None) -> torch.Tensor:
    """Concatenate every rank's row shard (in rank order) into a [total_rows, ...] tensor on
    every rank.  Shards may differ in size by one row; they are padded for the collective."""
    world = dist.get_world_size(group)
    shard = (total_rows + world - 1) // world
    dtype = local.dtype
    raw = local.contiguous().view(torch.uint8)   # bytes: every backend gathers uint8
    pad = torch.zeros((shard,) + tuple(raw.shape[1:]), dtype=torch.uint8, device=local.device)
    pad[: raw.shape[0]] = raw
    out = torch.empty((world * shard,) + tuple(raw.shape[1:]), dtype=torch.uint8, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    parts = []
    for r in range(world):
        s, e = row_shard(total_rows, world, r)
        parts.append(out[r * shard: r * shard + (e - s)])
    return torch.cat(parts, 0).view(dtype)


def global_mismatch(local_count: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of the ranks' Freivalds rejected-row counters (in place); 0 means every rank's
    every product verified."""
    dist.all_reduce(local_count, op=dist.ReduceOp.SUM, group=group)
    return local_count


def global_class_presence(masks: torch.Tensor, group=None) -> torch.Tensor:
    """OR of every rank's class-presence bitmasks [packs, words] (int32, as
    hawkeye_freivalds.class_presence returns them).  A row-sharded class-count run needs the
    global per-pack class lists: they fix which checkable products exist and their layout
    (the output does not depend on them).  NCCL has no bitwise reduction, so the masks
    (64 bytes per pack) are gathered and OR-ed locally."""
    world = dist.get_world_size(group)
    local = masks.contiguous()
    gathered = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(gathered, local, group=group)
    gathered = gathered.view((world,) + tuple(local.shape))
    out = gathered[0].clone()
    for r in range(1, world):
        out |= gathered[r]
    return out


def sharded_class_count_stats(
    x_shard: torch.Tensor,
    w_fp8: torch.Tensor,
    group=None,
    *,
    products_per_group: int = 32,
    class_chunk: int = 32,
    packed_count_lanes: int = 1,
    packed_group_lanes: int = 1,
):
    """HawkeyeFreivaldsStats of the unsharded product x @ w^T, evaluated on every rank of a
    row-sharded run (x_shard is this rank's rows, w the replicated weight)."""
    from . import hawkeye_freivalds as hf

    width = products_per_group * (packed_group_lanes if packed_group_lanes > 1 else 1)
    a = global_class_presence(hf.class_presence(x_shard, width), group)
    b = hf.class_presence(w_fp8, width)
    return hf.class_count_stats(
        hf._popcounts(a), hf._popcounts(b), int(w_fp8.shape[1]), products_per_group=products_per_group,
        class_chunk=class_chunk, packed_count_lanes=packed_count_lanes, packed_group_lanes=packed_group_lanes,
    )


def combine_freivalds_partials(partial: torch.Tensor, group=None) -> torch.Tensor:
    """Wrapping int64 SUM (in place) of per-rank partial Freivalds vectors.  With the weight
    column-sharded, rank r holds C[:, cols_r] and W[cols_r]; one global check A (W^T r) == C r
    needs sum_r W[cols_r]^T r[cols_r] ([K]) and sum_r C[:, cols_r] r[cols_r] ([M]).  (Each rank's
    block is also a complete product of its own, which the local row pass verifies.)"""
    if partial.dtype != torch.int64:
        raise RuntimeError("Freivalds partials must be int64")
    dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
