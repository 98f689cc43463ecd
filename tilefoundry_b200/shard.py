"""Candidate sharding across the GPUs of one node.

Candidates are independent, so a batch is split into contiguous ranges, one per rank
(one process per GPU), with the problem and frame tables replicated on every device.
The only exchange is the final gather of each candidate's results to one rank: over
``torch.distributed`` (NCCL between GPUs, gloo for CPU processes) as ``(verdict, makespan,
ii)`` in 12 bytes per candidate or packed as an int8 verdict and an int32 makespan in 5, or
(:class:`PeerGather`) by copy engines writing the packed results straight into rank 0's
memory, which leaves rank 0's SMs to the verifier.
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


__all__ = ["PeerGather", "gather_packed", "gather_results", "pack_results", "shard_bounds", "unpack_results"]


class PeerGather:
    """Every rank's packed results pushed into rank 0's memory by copy engines.

    The NCCL gather runs kernels on rank 0 that need SMs the verifier's persistent kernels
    occupy, so rank 0 verifies slower while it receives. Here rank 0 allocates ``slots``
    receive buffers of ``world x nbytes`` once (cudaMalloc) and exports them as CUDA IPC
    handles; every other rank maps them from its own device (peer access over NVLink) and
    copies its payload with cudaMemcpyAsync on a side stream, ordered after an event of the
    producing stream. No kernel reads another GPU's memory. One process per GPU of one node;
    the handles are exchanged once through ``torch.distributed``.

    ``send(slot, payload, stream)`` queues the copy of this rank's ``payload`` (uint8 CUDA
    tensor of at most ``nbytes``) into row ``rank`` of receive buffer ``slot`` after the work
    queued so far on ``stream``, and makes the next use of ``payload`` wait for it through
    ``wait(slot, stream)``. ``finish()`` waits for every copy of this rank; after a barrier
    rank 0 reads the rows with ``received(slot)``.
    """

    def __init__(self, nbytes: int, slots: int = 2, group=None) -> None:
        import torch
        import torch.distributed as dist
        from cuda.bindings import runtime as rt

        self._rt = rt
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = int(nbytes)
        self.slots = int(slots)
        self.device = torch.cuda.current_device()
        self.stream = torch.cuda.Stream(self.device)
        self._done = [torch.cuda.Event() for _ in range(self.slots)]
        self._sent = [False] * self.slots
        self._buffers: list[int] = []
        self._mapped: list[int] = []
        handles = None
        if self.rank == 0:
            handles = []
            for _ in range(self.slots):
                err, ptr = rt.cudaMalloc(self.world * self.nbytes)
                self._check(err, "cudaMalloc")
                self._buffers.append(int(ptr))
                err, handle = rt.cudaIpcGetMemHandle(ptr)
                self._check(err, "cudaIpcGetMemHandle")
                handles.append(bytes(handle.reserved))
        box = [handles]
        dist.broadcast_object_list(box, src=0, group=group)
        if self.rank != 0:
            for raw in box[0]:
                handle = rt.cudaIpcMemHandle_t()
                handle.reserved = raw
                err, ptr = rt.cudaIpcOpenMemHandle(handle, rt.cudaIpcMemLazyEnablePeerAccess)
                self._check(err, "cudaIpcOpenMemHandle")
                self._mapped.append(int(ptr))

    @staticmethod
    def _check(err, what: str) -> None:
        from cuda.bindings import runtime as rt

        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"{what} failed: {err}")

    def wait(self, slot: int, stream) -> None:
        """Make ``stream`` wait until this rank's last copy from ``slot`` has read its payload."""
        if self._sent[slot]:
            stream.wait_event(self._done[slot])

    def send(self, slot: int, payload, stream) -> None:
        """Queue this rank's payload for row ``rank`` of receive buffer ``slot``."""
        import torch

        nbytes = int(payload.numel())
        if nbytes > self.nbytes:
            raise ValueError("payload larger than the receive rows")
        ready = torch.cuda.Event()
        ready.record(stream)
        self.stream.wait_event(ready)
        if self.rank == 0:
            dst = self._buffers[slot]
        else:
            dst = self._mapped[slot]
        err, = self._rt.cudaMemcpyAsync(dst + self.rank * self.nbytes, payload.data_ptr(), nbytes,
                                        self._rt.cudaMemcpyKind.cudaMemcpyDefault,
                                        self._rt.cudaStream_t(self.stream.cuda_stream))
        self._check(err, "cudaMemcpyAsync")
        self._done[slot].record(self.stream)
        self._sent[slot] = True

    def finish(self) -> None:
        """Wait for every copy this rank queued."""
        self.stream.synchronize()

    def received(self, slot: int):
        """Rank 0: a uint8 tensor [world, nbytes] copy of receive buffer ``slot``."""
        import torch

        if self.rank != 0:
            raise RuntimeError("only rank 0 holds the receive buffers")
        out = torch.empty((self.world, self.nbytes), dtype=torch.uint8, device=torch.device("cuda", self.device))
        err, = self._rt.cudaMemcpy(out.data_ptr(), self._buffers[slot], self.world * self.nbytes,
                                   self._rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
        self._check(err, "cudaMemcpy")
        return out

    def close(self) -> None:
        """Unmap (other ranks) and free (rank 0) the receive buffers; every rank calls it after a barrier."""
        self.stream.synchronize()
        for ptr in self._mapped:
            self._rt.cudaIpcCloseMemHandle(ptr)
        self._mapped = []
        for ptr in self._buffers:
            self._rt.cudaFree(ptr)
        self._buffers = []
