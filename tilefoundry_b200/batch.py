"""Packers from schedules to the flat arrays of the C ABI.

A candidate schedule (``WarpgroupSchedule``, model.py:481) is split into

* its **frame** — lanes and sync edges, i.e. everything but the times. Frames are
  deduplicated: a batch of neighbourhood candidates that only move times shares one
  frame, so lane coverage, ownership, register locality and the lane/sync reachability
  of every required relation are analysed once per frame on the GPU;
* its **times**, either compact periodic (``PeriodicBatch``: per-op int16 deltas of the
  prologue and body offset starts plus an II, solve.py:206-231) or explicit rows
  (``RowsBatch``: start/issue_end/completion per iteration and operation).

Host-side work here is limited to what the dense device layout cannot express: the
record-constructor rules on ids and duplicates (class 1), lanes naming unknown
operations (class 4) and rows outside the ``[0, I) x ops`` grid (class 7).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib
from .model import is_identifier
from .problem import PackedProblem

_ABSENT = _lib.TFV_LANE_ABSENT << _lib.TFV_LANE_SHIFT
_INT32_MIN, _INT32_MAX = -(2**31), 2**31 - 1


def _is_int(value: object) -> bool:
    return type(value) is int or isinstance(value, np.integer)


def schedule_parts(schedule: object) -> tuple[list, list, list]:
    """``(lanes, sync, rows)`` of a schedule record (the reference's or the mirror's) or a raw triple."""
    if isinstance(schedule, tuple) and len(schedule) == 3:
        return schedule  # type: ignore[return-value]
    lanes = [list(lane.operations) for lane in schedule.lanes]  # type: ignore[attr-defined]
    sync = [(e.after, e.before, e.distance) for e in schedule.sync]  # type: ignore[attr-defined]
    rows = [(t.iteration, t.operation_id, t.start, t.issue_end, t.completion) for t in schedule.times]  # type: ignore[attr-defined]
    return lanes, sync, rows


class FrameSet:
    """Deduplicated frames (lanes + sync set) of one problem, as host arrays."""

    def __init__(self, packed: PackedProblem) -> None:
        self.packed = packed
        self._frame_index: dict[tuple, int] = {}
        self._set_index: dict[tuple, int] = {}
        self.lane_pos: list[np.ndarray] = []
        self.lane_count: list[int] = []
        self.flags: list[int] = []
        self.sync_set: list[int] = []
        self.sync_offsets: list[int] = [0]
        self.sync_edges: list[tuple[int, int, int]] = []
        self.frames: list[tuple[tuple, tuple]] = []

    def __len__(self) -> int:
        return len(self.lane_count)

    def add(self, lanes, sync) -> int:
        """Index of the frame with these lanes and sync edges (added when new)."""
        lanes_t = tuple(tuple(lane) for lane in lanes)
        sync_t = tuple(tuple(edge) for edge in sync)
        key = (lanes_t, sync_t)
        found = self._frame_index.get(key)
        if found is not None:
            return found
        packed = self.packed
        flags = 0
        # Lane programs (WarpgroupLane / WarpgroupSchedule constructors, model.py:431-499).
        seen: set[str] = set()
        if not lanes_t:
            flags |= _lib.TFV_FRAME_MALFORMED
        pos = np.full(packed.n_ops, _ABSENT, dtype=np.uint16)
        for lane_index, lane in enumerate(lanes_t):
            if len(set(lane)) != len(lane):
                flags |= _lib.TFV_FRAME_MALFORMED
            position = 0
            for op in lane:
                if not is_identifier(op):
                    flags |= _lib.TFV_FRAME_MALFORMED
                    continue
                if op in seen:
                    flags |= _lib.TFV_FRAME_MALFORMED
                    continue
                seen.add(op)
                k = packed.index.get(op)
                if k is None:
                    flags |= _lib.TFV_FRAME_UNKNOWN_LANE_OP
                    continue
                if lane_index < _lib.TFV_MAX_LANES:
                    pos[k] = (lane_index << _lib.TFV_LANE_SHIFT) | position
                    position += 1
        # Sync edges (SynchronizationEdge constructor, model.py:450-455), sorted (model.py:506).
        valid_edges = []
        for edge in sync_t:
            if len(edge) != 3:
                flags |= _lib.TFV_FRAME_MALFORMED
                continue
            after, before, distance = edge
            if not (is_identifier(after) and is_identifier(before) and _is_int(distance) and distance >= 0):
                flags |= _lib.TFV_FRAME_MALFORMED
                continue
            if after == before and distance == 0:
                flags |= _lib.TFV_FRAME_MALFORMED
            valid_edges.append((after, before, int(distance)))
        if len(set(valid_edges)) != len(valid_edges):
            flags |= _lib.TFV_FRAME_MALFORMED
        ordered = tuple(sorted(valid_edges))
        set_id = self._set_index.get(ordered)
        if set_id is None:
            set_id = len(self.sync_offsets) - 1
            self._set_index[ordered] = set_id
            for after, before, distance in ordered:
                self.sync_edges.append(
                    (packed.index.get(after, -1), packed.index.get(before, -1), min(distance, _lib.TFV_TIME_LIMIT))
                )
            self.sync_offsets.append(len(self.sync_edges))
        frame_id = len(self.lane_count)
        self._frame_index[key] = frame_id
        self.lane_pos.append(pos)
        self.lane_count.append(len(lanes_t))
        self.flags.append(flags)
        self.sync_set.append(set_id)
        self.frames.append(key)
        return frame_id

    def arrays(self) -> dict[str, np.ndarray]:
        """Host arrays in the layout of ``tfv_frames``."""
        n = self.packed.n_ops
        lane_pos = np.stack(self.lane_pos) if self.lane_pos else np.zeros((0, n), dtype=np.uint16)
        edges = np.array(self.sync_edges, dtype=np.int32).reshape(-1, 3)
        return {
            "lane_pos": np.ascontiguousarray(lane_pos, dtype=np.uint16),
            "lane_count": np.array(self.lane_count, dtype=np.int32),
            "flags": np.array(self.flags, dtype=np.int32),
            "sync_set": np.array(self.sync_set, dtype=np.int32),
            "sync_offsets": np.array(self.sync_offsets, dtype=np.int32),
            "sync_edges": edges if edges.size else np.zeros((1, 3), dtype=np.int32),
        }


@dataclass
class PeriodicBatch:
    """Compact periodic candidates: int16 deltas against per-op base starts, op-major."""

    base_prologue: np.ndarray  # [N] int32
    base_offset: np.ndarray  # [N] int32
    prologue_delta: np.ndarray  # [N, n] int16
    offset_delta: np.ndarray  # [N, n] int16
    ii: np.ndarray  # [n] int32
    frame: np.ndarray  # [n] int32

    @property
    def n(self) -> int:
        return int(self.ii.shape[0])

    @classmethod
    def from_starts(cls, prologue, offset, ii, frame, base_prologue=None, base_offset=None) -> "PeriodicBatch":
        """Build from absolute starts ``prologue``/``offset`` of shape [n, N].

        The base defaults to the per-operation midpoint of each column; every delta
        must fit int16.
        """
        prologue = np.asarray(prologue, dtype=np.int64)
        offset = np.asarray(offset, dtype=np.int64)
        if base_prologue is None:
            base_prologue = (prologue.min(axis=0) + prologue.max(axis=0)) // 2
        if base_offset is None:
            base_offset = (offset.min(axis=0) + offset.max(axis=0)) // 2
        base_prologue = np.asarray(base_prologue, dtype=np.int64)
        base_offset = np.asarray(base_offset, dtype=np.int64)
        dp = prologue - base_prologue[None, :]
        dq = offset - base_offset[None, :]
        for name, delta in (("prologue", dp), ("offset", dq)):
            if delta.size and (delta.min() < -32768 or delta.max() > 32767):
                raise ValueError(f"{name} starts span more than the int16 delta range around their base")
        for name, base in (("prologue", base_prologue), ("offset", base_offset)):
            if base.size and np.abs(base).max() >= _lib.TFV_BASE_LIMIT:
                raise ValueError(f"{name} base starts must lie in (-2^28, 2^28)")
        return cls(
            base_prologue=base_prologue.astype(np.int32),
            base_offset=base_offset.astype(np.int32),
            prologue_delta=np.ascontiguousarray(dp.T.astype(np.int16)),
            offset_delta=np.ascontiguousarray(dq.T.astype(np.int16)),
            ii=np.ascontiguousarray(np.asarray(ii, dtype=np.int64).astype(np.int32)),
            frame=np.ascontiguousarray(np.asarray(frame, dtype=np.int64).astype(np.int32)),
        )


def periodic_groups(prologue, offset, ii, frame) -> list[tuple[np.ndarray, PeriodicBatch]]:
    """Split candidates given by absolute starts into batches whose deltas fit int16.

    ``prologue``/``offset`` are [n, N] starts (any integers), ``ii`` and ``frame`` [n]. The
    first batch takes every candidate within the int16 range of the per-operation midpoint
    of all candidates (the base :meth:`PeriodicBatch.from_starts` picks); each further batch
    is based on the starts of the first candidate left and takes every remaining candidate
    within range of that base. So a batch with a few outliers becomes one main batch plus a
    batch per cluster of outliers, and every candidate gets a verdict. A base outside
    (-2^28, 2^28) makes its batch's candidates report TFV_CLASS_OUT_OF_RANGE, as the kernels
    do for any base out of that domain. Returns ``(candidate indices, batch)`` pairs that
    cover every candidate once, in increasing index order within each batch.
    """
    prologue = np.asarray(prologue, dtype=np.int64)
    offset = np.asarray(offset, dtype=np.int64)
    ii = np.asarray(ii, dtype=np.int64)
    frame = np.asarray(frame, dtype=np.int64)
    n = prologue.shape[0]
    left = np.arange(n)
    groups: list[tuple[np.ndarray, PeriodicBatch]] = []
    first = True
    while left.size:
        p, o = prologue[left], offset[left]
        if first:
            bp = (p.min(axis=0) + p.max(axis=0)) // 2
            bo = (o.min(axis=0) + o.max(axis=0)) // 2
        else:  # the first remaining candidate fits its own base
            bp, bo = p[0].copy(), o[0].copy()
        fits = ((np.abs(p - bp[None, :]) <= 32767).all(axis=1) & (np.abs(o - bo[None, :]) <= 32767).all(axis=1))
        first = False
        if not fits.any():
            continue
        take = left[fits]
        clip = lambda base: np.clip(base, -(2**31), 2**31 - 1)  # noqa: E731 (int32 storage of any base)
        dp = (prologue[take] - bp[None, :]).T
        dq = (offset[take] - bo[None, :]).T
        groups.append((take, PeriodicBatch(
            base_prologue=clip(bp).astype(np.int32), base_offset=clip(bo).astype(np.int32),
            prologue_delta=np.ascontiguousarray(dp.astype(np.int16)),
            offset_delta=np.ascontiguousarray(dq.astype(np.int16)),
            ii=np.ascontiguousarray(np.clip(ii[take], -(2**31), 2**31 - 1).astype(np.int32)),
            frame=np.ascontiguousarray(frame[take].astype(np.int32)),
        )))
        left = left[~fits]
    return groups


@dataclass
class RowsBatch:
    """Explicit timing rows [n, I, N] plus the host-side facts the dense layout cannot hold."""

    start: np.ndarray
    issue_end: np.ndarray
    completion: np.ndarray
    frame: np.ndarray
    row_flags: np.ndarray
    # makespan / II of flagged candidates, taken over every row the schedule lists
    override: np.ndarray  # [n] bool
    override_makespan: np.ndarray
    override_ii: np.ndarray

    @property
    def n(self) -> int:
        return int(self.frame.shape[0])


def _row_ok(row) -> bool:
    """TimedOperation constructor rules (model.py:468-477)."""
    if len(row) != 5:
        return False
    iteration, op, start, issue_end, completion = row
    return (
        _is_int(iteration) and iteration >= 0 and is_identifier(op)
        and _is_int(start) and _is_int(issue_end) and _is_int(completion)
        and start >= 0 and issue_end > 0 and completion > 0 and issue_end > start and completion >= issue_end
    )


def pack_rows(packed: PackedProblem, frames: FrameSet, schedules) -> RowsBatch:
    """Pack schedules (records or ``(lanes, sync, rows)`` triples) into a rows batch."""
    N, I = packed.n_ops, packed.iterations
    n = len(schedules)
    start = np.zeros((n, I, N), dtype=np.int32)
    issue_end = np.ones((n, I, N), dtype=np.int32)
    completion = np.ones((n, I, N), dtype=np.int32)
    frame = np.zeros(n, dtype=np.int32)
    row_flags = np.zeros(n, dtype=np.int32)
    override = np.zeros(n, dtype=bool)
    override_makespan = np.zeros(n, dtype=np.int32)
    override_ii = np.zeros(n, dtype=np.int32)
    first_op = packed.op_ids[0]
    limit = _lib.TFV_TIME_LIMIT
    for c, schedule in enumerate(schedules):
        lanes, sync, rows = schedule_parts(schedule)
        frame[c] = frames.add(lanes, sync)
        flags = 0
        present = np.zeros((I, N), dtype=bool)
        seen: set[tuple] = set()
        for row in rows:
            if not _row_ok(row):
                flags |= _lib.TFV_ROWS_MALFORMED
            if len(row) != 5:
                continue
            iteration, op, s, e, cp = row
            key = (iteration, op)
            if key in seen:
                flags |= _lib.TFV_ROWS_MALFORMED
                continue
            seen.add(key)
            k = packed.index.get(op) if isinstance(op, str) else None
            if k is None or not _is_int(iteration) or not (0 <= iteration < I):
                flags |= _lib.TFV_ROWS_COVERAGE
                continue
            if not (_is_int(s) and _is_int(e) and _is_int(cp)):
                continue
            if _row_ok(row) and max(s, e, cp) >= limit:
                s, e, cp = limit, limit + 1, limit + 1  # keeps the verdict "out of range"
            start[c, iteration, k] = min(max(s, _INT32_MIN), _INT32_MAX)
            issue_end[c, iteration, k] = min(max(e, _INT32_MIN), _INT32_MAX)
            completion[c, iteration, k] = min(max(cp, _INT32_MIN), _INT32_MAX)
            present[iteration, k] = True
        if not present.all():
            flags |= _lib.TFV_ROWS_COVERAGE
            filled = np.argwhere(present)
            if len(filled):  # missing instances repeat a listed row: no new verdict or makespan
                i0, k0 = filled[0]
                start[c][~present] = start[c, i0, k0]
                issue_end[c][~present] = issue_end[c, i0, k0]
                completion[c][~present] = completion[c, i0, k0]
        row_flags[c] = flags
        if flags:
            ints = [r for r in rows if len(r) == 5 and _is_int(r[4])]
            mk = max((int(r[4]) for r in ints), default=0)
            starts = {(r[0], r[1]): r[2] for r in ints if _is_int(r[2])}
            iiv = 0
            if I >= 3 and (2, first_op) in starts and (1, first_op) in starts:
                iiv = int(starts[(2, first_op)]) - int(starts[(1, first_op)])
            override[c] = True
            override_makespan[c] = min(max(mk, _INT32_MIN), _INT32_MAX)
            override_ii[c] = min(max(iiv, _INT32_MIN), _INT32_MAX)
    return RowsBatch(start, issue_end, completion, frame, row_flags, override, override_makespan, override_ii)


__all__ = ["FrameSet", "PeriodicBatch", "RowsBatch", "pack_rows", "periodic_groups", "schedule_parts"]
