"""Neighbourhood search with the GPU as the bulk oracle.

The reference's solver (solve.py:234-512) builds a CP-SAT model of the periodic body,
minimises the II and then the makespan at that II (solve.py:452, 467), and exports the
incumbent (sync.py:21-62). This module is the GPU side of that loop: given an incumbent
in periodic form, it draws a batch of seeded neighbours (tighter IIs, operations pulled
earlier, lane moves), verifies the whole batch on the GPU with the exact verifier, and
keeps the best valid neighbour by the solver's objective (II first, then makespan).
Every accepted schedule is a verified schedule; the search never trusts a heuristic.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import numpy as np

from .batch import FrameSet, PeriodicBatch
from .model import SCHEDULE_FORMAT, TimedOperation, WarpgroupLane, WarpgroupSchedule, WarpgroupSolveResult
from .verify import _verifier_for
from .workloads import Witness


@dataclass
class SearchResult:
    """The best verified schedule found and the search's bookkeeping."""

    witness: Witness
    ii: int
    makespan: int
    evaluated: int = 0
    accepted: int = 0
    history: list[tuple[int, int]] = field(default_factory=list)  # (ii, makespan) after each round

    def solve_result(self, packed: Any) -> WarpgroupSolveResult:
        """The schedule as the solver's result record (rows of solve.py:206-231)."""
        times = []
        for i in range(packed.iterations):
            for k, op in enumerate(packed.op_ids):
                start = int(self.witness.prologue[k]) if i == 0 else int(self.witness.offset[k]) + i * self.witness.ii
                times.append(TimedOperation(i, op, start, start + int(packed.issue[k]), start + int(packed.latency[k])))
        return WarpgroupSolveResult(
            "FEASIBLE_NOT_PROVEN",
            tuple(WarpgroupLane(tuple(lane)) for lane in self.witness.lanes),
            tuple(times),
            self.witness.ii if packed.iterations >= 3 else None,
        )

    def schedule(self, packed: Any) -> WarpgroupSchedule:
        """The schedule record with the witness's own sync edges."""
        result = self.solve_result(packed)
        from .model import SynchronizationEdge

        return WarpgroupSchedule(
            SCHEDULE_FORMAT, result.lanes, tuple(SynchronizationEdge(*e) for e in self.witness.sync), result.times
        )


def _objective(ii: np.ndarray, makespan: np.ndarray, iterations: int) -> np.ndarray:
    """Lexicographic (II, makespan) as one int64 key; the II only counts with I >= 3."""
    lead = ii.astype(np.int64) if iterations >= 3 else np.zeros_like(ii, dtype=np.int64)
    return lead * (1 << 32) + makespan.astype(np.int64)


def _lane_moves(packed, incumbent: Witness, rng: np.random.Generator, count: int = 16) -> FrameSet:
    """The incumbent's frame (index 0) and ``count`` frames with one operation moved to a
    random position of a random lane."""
    N = packed.n_ops
    frames = FrameSet(packed)
    frames.add(incumbent.lanes, incumbent.sync)
    for _ in range(count):
        lanes = [list(lane) for lane in incumbent.lanes]
        op = packed.op_ids[int(rng.integers(N))]
        for lane in lanes:
            if op in lane:
                lane.remove(op)
        target = lanes[int(rng.integers(len(lanes)))]
        target.insert(int(rng.integers(len(target) + 1)), op)
        frames.add(lanes, incumbent.sync)
    return frames


def _device_neighbours(torch, incumbent: Witness, n: int, n_frames: int, gen, step: int, dev):
    """Seeded neighbours of the incumbent drawn on the device, as a periodic batch of device
    tensors with the incumbent's starts as base (nothing crosses the host link).

    Kinds: (0) a tighter II with the same offsets; (1) up to three operations pulled earlier
    in the body (and half the time in the prologue); (2) a tighter II with operations pulled
    earlier; (3) one of the lane-move frames, times kept.
    """
    N = int(incumbent.prologue.shape[0])
    i64 = dict(dtype=torch.int64, device=dev)
    kind = torch.randint(0, 4, (n,), generator=gen, **i64)
    cut = torch.randint(1, max(2, step) + 1, (n,), generator=gen, **i64)
    tighter = (kind == 0) | (kind == 2)
    ii = torch.full((n,), int(incumbent.ii), **i64) - torch.where(tighter, cut, 0)
    dp = torch.zeros((N, n), **i64)
    dq = torch.zeros((N, n), **i64)
    pulled = (kind == 1) | (kind == 2)
    cols = torch.arange(n, device=dev)
    for _ in range(3):
        ops = torch.randint(0, N, (n,), generator=gen, **i64)
        pull = torch.randint(1, max(2, step) + 1, (n,), generator=gen, **i64) * pulled
        half = torch.rand((n,), generator=gen, device=dev) < 0.5
        dp.index_put_((ops, cols), -torch.where(half, pull, 0), accumulate=True)
        dq.index_put_((ops, cols), -pull, accumulate=True)
    frame = torch.where(kind == 3, torch.randint(1, max(2, n_frames), (n,), generator=gen, **i64), 0)
    ii = ii.clamp(min=1)
    # every materialised start stays representable and non-negative before the verifier sees it
    base_p = torch.as_tensor(incumbent.prologue, **i64)
    base_o = torch.as_tensor(incumbent.offset, **i64)
    dp = torch.maximum(dp, -base_p[:, None]).clamp(-32768, 32767)
    dq = torch.maximum(dq, -(base_o[:, None] + ii[None, :])).clamp(-32768, 32767)
    return {
        "base_prologue": base_p.to(torch.int32),
        "base_offset": base_o.to(torch.int32),
        "prologue_delta": dp.to(torch.int16).contiguous(),
        "offset_delta": dq.to(torch.int16).contiguous(),
        "ii": ii.to(torch.int32),
        "frame": frame.to(torch.int32),
    }


def improve_periodic(
    problem: Any,
    incumbent: Witness,
    *,
    rounds: int = 20,
    batch: int = 1 << 16,
    seed: int = 0,
    device: int = 0,
) -> SearchResult:
    """Descend on (II, makespan) from a verified periodic incumbent.

    Each round draws ``batch`` neighbours on the GPU, verifies them there with the exact
    verifier, picks the best valid one by the solver's objective on the device, and moves
    to it when it improves the incumbent; only the lane-move frames go to the device and
    only the winner's starts come back. The step size adapts to the incumbent's II. The
    incumbent itself must verify.
    """
    import torch

    verifier = _verifier_for(problem, device)
    packed = verifier.packed
    rng = np.random.default_rng(seed)
    dev = torch.device("cuda", verifier.device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    frames = FrameSet(packed)
    f0 = frames.add(incumbent.lanes, incumbent.sync)
    start = PeriodicBatch.from_starts(incumbent.prologue[None, :], incumbent.offset[None, :],
                                      np.array([incumbent.ii]), np.array([f0]))
    verdict, makespan, ii = verifier.verify_periodic(frames, start)
    if verdict[0] != 0:
        raise ValueError(f"the incumbent does not verify (class {int(verdict[0])})")
    result = SearchResult(incumbent, int(incumbent.ii), int(makespan[0]))
    best_key = int(_objective(np.array([result.ii]), np.array([result.makespan]), packed.iterations)[0])
    lead = 1 if packed.iterations >= 3 else 0
    for _ in range(rounds):
        step = max(1, result.ii // 16)
        nframes = _lane_moves(packed, result.witness, rng)
        dframes = verifier.frames_to_device(nframes)
        table = verifier.analyze(dframes)
        cand = _device_neighbours(torch, result.witness, batch, len(nframes), gen, step, dev)
        verdict_d, makespan_d, _ii = verifier.verify_periodic_device(dframes, table, cand)
        result.evaluated += batch
        keys = cand["ii"].to(torch.int64) * lead * (1 << 32) + makespan_d.to(torch.int64)
        keys = torch.where(verdict_d == 0, keys, torch.iinfo(torch.int64).max)
        j = int(torch.argmin(keys).item())
        key = int(keys[j].item())
        if key < best_key and int(verdict_d[j].item()) == 0:
            best_key = key
            lanes, sync = nframes.frames[int(cand["frame"][j].item())]
            p = cand["base_prologue"].to(torch.int64) + cand["prologue_delta"][:, j].to(torch.int64)
            o = cand["base_offset"].to(torch.int64) + cand["offset_delta"][:, j].to(torch.int64)
            result.witness = Witness([list(lane) for lane in lanes], [tuple(edge) for edge in sync],
                                     p.cpu().numpy(), o.cpu().numpy(), int(cand["ii"][j].item()))
            result.ii = result.witness.ii
            result.makespan = int(makespan_d[j].item())
            result.accepted += 1
        result.history.append((result.ii, result.makespan))
    return result


__all__ = ["SearchResult", "improve_periodic"]
