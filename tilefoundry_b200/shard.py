"""Candidate sharding across the GPUs of one node.

Candidates are independent, so a batch is split into contiguous ranges, one per rank
(one process per GPU), with the problem and frame tables replicated on every device.
The only exchange is the final gather of each candidate's results to one rank over
``torch.distributed`` (NCCL between GPUs, gloo for CPU processes): ``(verdict, makespan,
ii)`` as 12 bytes per candidate, or packed as an int8 verdict and an int32 makespan in 5.
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


def pack_results(verdict, makespan, out=None):
    """``(verdict, makespan)`` of one shard as one uint8 tensor of 5 bytes per candidate.

    The makespans come first as int32 (4 bytes each), then the verdicts as int8: every
    verdict class, -4 to 21, fits. The II is left out: a periodic candidate's II is its
    input II (0 below three iterations), which the batch's producer holds. ``out`` may be
    a preallocated uint8 tensor of ``5 * n`` bytes whose first ``4 * n`` bytes already hold
    the makespans (written there by the verifier); then only the verdicts are converted.
    """
    import torch

    n = int(verdict.numel())
    if out is None:
        out = torch.empty(5 * n, dtype=torch.uint8, device=verdict.device)
    mk = out[: 4 * n].view(torch.int32)
    if mk.data_ptr() != makespan.data_ptr():
        mk.copy_(makespan.reshape(-1))
    out[4 * n:].view(torch.int8).copy_(verdict.reshape(-1))
    return out


def unpack_results(packed, n: int):
    """Inverse of :func:`pack_results`: int32 ``(verdict, makespan)`` tensors of ``n``."""
    import torch

    makespan = packed[: 4 * n].view(torch.int32).clone()
    verdict = packed[4 * n: 5 * n].view(torch.int8).to(torch.int32)
    return verdict, makespan


def gather_packed(packed, n_total: int, *, dst: int = 0, group=None):
    """Gather every rank's :func:`pack_results` tensor to ``dst``: int32 ``(verdict,
    makespan)`` of all ``n_total`` candidates there, None elsewhere. 5 bytes per candidate
    cross the interconnect instead of 12."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = [shard_bounds(n_total, r, world) for r in range(world)]
    widest = max(hi - lo for lo, hi in sizes)
    padded = torch.zeros(5 * widest, dtype=torch.uint8, device=packed.device)
    padded[: packed.numel()] = packed
    pieces = [torch.empty_like(padded) for _ in range(world)] if rank == dst else None
    dist.gather(padded, gather_list=pieces, dst=dst, group=group)
    if rank != dst:
        return None
    verdicts, makespans = [], []
    for r, (lo, hi) in enumerate(sizes):
        m = hi - lo
        piece = pieces[r]
        # the shard was packed for m candidates: makespans in its first 4m bytes, verdicts next
        makespans.append(piece[: 4 * m].view(torch.int32))
        verdicts.append(piece[4 * m: 5 * m].view(torch.int8).to(torch.int32))
    return torch.cat(verdicts), torch.cat(makespans)


__all__ = ["gather_packed", "gather_results", "pack_results", "shard_bounds", "unpack_results"]
