"""Data-parallel sharding of independent depth units (images, or multi-view scenes)
over the ranks of one node, and the optional gather of depth maps to rank 0.

The depth path has no exchange step: each GPU holds a full weight replica and runs
its contiguous slice of the units (one process per GPU). A scene's views stay on
one rank, because global attention couples them. The only collective is the optional
gather of the finished depth maps (equal-sized slabs over NCCL on NVLink; gloo on
CPU in the tests).
"""
from __future__ import annotations


def shard_range(n_units: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [first, end) slice of n_units for `rank`: the first n_units % world
    ranks take one extra unit, so slice sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_units < 0:
        raise ValueError("negative unit count")
    base, extra = divmod(n_units, world)
    first = rank * base + min(rank, extra)
    return first, first + base + (1 if rank < extra else 0)


def shard_counts(n_units: int, world: int) -> list[int]:
    return [e - f for f, e in (shard_range(n_units, world, r) for r in range(world))]


def scene_views(n_scenes: int, views_per_scene: int, world: int, rank: int) -> tuple[int, int]:
    """View slice [first, end) of a rank when whole scenes are sharded."""
    f, e = shard_range(n_scenes, world, rank)
    return f * views_per_scene, e * views_per_scene


def gather_to_rank0(local, n_units: int, group=None):
    """Gathers every rank's [count, ...] tensor slice into one [n_units, ...] tensor on
    rank 0 (None elsewhere). Slices are padded to the largest shard so the collective
    moves equal-sized slabs (all_gather); every rank takes the same collective steps.
    `local` lives on the device the process group's backend uses."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    counts = shard_counts(n_units, world)
    if local.shape[0] != counts[rank]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} units, expected {counts[rank]}")
    cap = max(counts)
    slab = local
    if local.shape[0] < cap:
        slab = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        slab[: local.shape[0]] = local
    slabs = [torch.empty_like(slab) for _ in range(world)]
    dist.all_gather(slabs, slab.contiguous(), group=group)
    if rank != 0:
        return None
    return torch.cat([s[:c] for s, c in zip(slabs, counts)], 0)
