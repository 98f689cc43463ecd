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


def _neighbours(packed, incumbent: Witness, n: int, rng: np.random.Generator, step: int):
    """Seeded neighbours of the incumbent, as deltas against its own starts.

    Kinds: (0) a tighter II with the same offsets; (1) a few operations pulled earlier in
    the prologue and the body; (2) a tighter II with the body offsets of late operations
    pulled earlier; (3) one operation moved to another lane position, times kept.
    """
    N = packed.n_ops
    frames = FrameSet(packed)
    base = frames.add(incumbent.lanes, incumbent.sync)
    moves = []
    for _ in range(16):
        lanes = [list(lane) for lane in incumbent.lanes]
        op = packed.op_ids[int(rng.integers(N))]
        for lane in lanes:
            if op in lane:
                lane.remove(op)
        target = lanes[int(rng.integers(len(lanes)))]
        target.insert(int(rng.integers(len(target) + 1)), op)
        moves.append(frames.add(lanes, incumbent.sync))
    kind = rng.integers(0, 4, size=n)
    dp = np.zeros((N, n), dtype=np.int64)
    dq = np.zeros((N, n), dtype=np.int64)
    ii = np.full(n, incumbent.ii, dtype=np.int64)
    frame = np.full(n, base, dtype=np.int32)
    cut = rng.integers(1, max(2, step) + 1, size=n)
    ii[(kind == 0) | (kind == 2)] -= cut[(kind == 0) | (kind == 2)]
    for sel in (kind == 1, kind == 2):
        cols = np.flatnonzero(sel)
        for _ in range(3):
            ops = rng.integers(0, N, size=cols.size)
            pull = rng.integers(1, max(2, step) + 1, size=cols.size)
            dp[ops, cols] -= np.where(rng.random(cols.size) < 0.5, pull, 0)
            dq[ops, cols] -= pull
    cols = np.flatnonzero(kind == 3)
    frame[cols] = np.array(moves, dtype=np.int32)[rng.integers(0, len(moves), size=cols.size)]
    # keep every materialised start representable and non-negative before the verifier sees it
    dp = np.maximum(dp, -incumbent.prologue[:, None])
    dq = np.maximum(dq, -(incumbent.offset[:, None] + np.maximum(ii, 1)[None, :]))
    batch = PeriodicBatch(
        base_prologue=incumbent.prologue.astype(np.int32),
        base_offset=incumbent.offset.astype(np.int32),
        prologue_delta=np.ascontiguousarray(np.clip(dp, -32768, 32767).astype(np.int16)),
        offset_delta=np.ascontiguousarray(np.clip(dq, -32768, 32767).astype(np.int16)),
        ii=np.maximum(ii, 1).astype(np.int32),
        frame=frame,
    )
    return frames, batch


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

    Each round verifies ``batch`` neighbours on the GPU and moves to the best valid one
    when it improves the objective; the step size adapts to the incumbent's II. The
    incumbent itself must verify.
    """
    verifier = _verifier_for(problem, device)
    packed = verifier.packed
    rng = np.random.default_rng(seed)
    frames = FrameSet(packed)
    f0 = frames.add(incumbent.lanes, incumbent.sync)
    start = PeriodicBatch.from_starts(incumbent.prologue[None, :], incumbent.offset[None, :],
                                      np.array([incumbent.ii]), np.array([f0]))
    verdict, makespan, ii = verifier.verify_periodic(frames, start)
    if verdict[0] != 0:
        raise ValueError(f"the incumbent does not verify (class {int(verdict[0])})")
    result = SearchResult(incumbent, int(incumbent.ii), int(makespan[0]))
    best_key = int(_objective(np.array([result.ii]), np.array([result.makespan]), packed.iterations)[0])
    for _ in range(rounds):
        step = max(1, result.ii // 16)
        nframes, cand = _neighbours(packed, result.witness, batch, rng, step)
        verdict, makespan, ii_out = verifier.verify_periodic(nframes, cand)
        result.evaluated += batch
        valid = np.flatnonzero(verdict == 0)
        if valid.size:
            keys = _objective(cand.ii[valid], makespan[valid], packed.iterations)
            j = int(valid[int(np.argmin(keys))])
            key = int(keys.min())
            if key < best_key:
                best_key = key
                lanes, sync = nframes.frames[int(cand.frame[j])]
                result.witness = Witness(
                    [list(lane) for lane in lanes],
                    [tuple(edge) for edge in sync],
                    cand.base_prologue.astype(np.int64) + cand.prologue_delta[:, j].astype(np.int64),
                    cand.base_offset.astype(np.int64) + cand.offset_delta[:, j].astype(np.int64),
                    int(cand.ii[j]),
                )
                result.ii = int(cand.ii[j])
                result.makespan = int(makespan[j])
                result.accepted += 1
        result.history.append((result.ii, result.makespan))
    return result


__all__ = ["SearchResult", "improve_periodic"]
