"""Candidate sharding across the GPUs of one node.

Candidates are independent, so a batch is split into contiguous ranges, one per rank
(one process per GPU), with the problem and frame tables replicated on every device.
The only exchange is the final gather of each candidate's ``(verdict, makespan, ii)``
to one rank — 12 bytes per candidate — over ``torch.distributed`` (NCCL between
GPUs, gloo for CPU processes).
"""

from __future__ import annotations


def shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous balanced range ``[start, stop)`` of ``n`` items for ``rank`` of ``world``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_results(results, n_total: int, *, dst: int = 0, group=None):
    """Gather every rank's ``(verdict, makespan, ii)`` shard to ``dst``.

    ``results`` are three equal-length int32 tensors (CUDA tensors with NCCL, CPU
    tensors with gloo) holding this rank's contiguous shard of ``n_total``
    candidates. Returns the full ``[3, n_total]`` tensor on ``dst`` and None elsewhere.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    widest = max(shard_bounds(n_total, r, world)[1] - shard_bounds(n_total, r, world)[0] for r in range(world))
    local = torch.stack([t.to(torch.int32) for t in results])
    padded = torch.zeros((3, widest), dtype=torch.int32, device=local.device)
    padded[:, : local.shape[1]] = local
    pieces = [torch.empty_like(padded) for _ in range(world)] if rank == dst else None
    dist.gather(padded, gather_list=pieces, dst=dst, group=group)
    if rank != dst:
        return None
    parts = []
    for r in range(world):
        lo, hi = shard_bounds(n_total, r, world)
        parts.append(pieces[r][:, : hi - lo])
    return torch.cat(parts, dim=1)


__all__ = ["gather_results", "shard_bounds"]
