"""Batch driver of the C oracle (test infrastructure only).

Prepares the integer tables of ``oracle/tfv_oracle.c`` from the oracle's own Python
restatement (:mod:`oracle.verify_port`) — never from the product's packer — and
classifies candidates with it. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use this module.

Two candidate forms are accepted:

* raw candidates ``(lanes, sync, rows)`` exactly as :func:`verify_port.classify`
  takes them (any schedule, including malformed ones);
* compact periodic candidates (``solve.py:206-231``): per-candidate prologue and
  offset starts plus an II, and a structure ("frame") index into a list of
  ``(lanes, sync)`` pairs.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

from . import verify_port as port

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_build" / "libtfv_oracle.so"

_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)


class _Problem(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_int), ("iters", ctypes.c_int), ("lanes", ctypes.c_int),
        ("issue", _i32p), ("lat", _i32p), ("wg", _i32p),
        ("n_rel", ctypes.c_int), ("rel", _i32p),
        ("n_car", ctypes.c_int), ("car", _i32p),
        ("n_reg", ctypes.c_int), ("reg_off", _i32p), ("reg_ops", _i32p),
        ("n_res", ctypes.c_int), ("cap", _i32p), ("win_off", _i32p), ("win_res", _i32p),
        ("win_amt", _i32p), ("win_dur", _i32p),
    ]


def build() -> Path:
    """Compile the C oracle with ``oracle/Makefile`` if it is missing or stale."""
    source = HERE / "tfv_oracle.c"
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < source.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


_lib = None


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIBRARY))
        lib.oracle_classify_batch.restype = None
        lib.oracle_classify_batch.argtypes = [
            ctypes.POINTER(_Problem), ctypes.c_int, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p,
            ctypes.c_longlong, _i32p, _i32p, _i64p, _i64p, _i64p, _i32p, ctypes.c_void_p, ctypes.c_void_p,
        ]
        _lib = lib
    return _lib


def _ptr(array: np.ndarray, kind=_i32p):
    return array.ctypes.data_as(kind)


class OracleProblem:
    """Integer tables of one problem, derived by :mod:`oracle.verify_port`."""

    def __init__(self, problem) -> None:
        ops = sorted(problem.loop.ops, key=lambda item: item.id)
        self.problem = problem
        self.op_ids = [op.id for op in ops]
        self.index = {op_id: k for k, op_id in enumerate(self.op_ids)}
        self.n = len(ops)
        self.iterations = problem.loop.iterations
        self.lanes = problem.warp_groups
        self.issue = np.array([op.issue_duration for op in ops], dtype=np.int32)
        self.latency = np.array([op.completion_latency for op in ops], dtype=np.int32)
        self.wg = np.array([-1 if op.warp_group is None else op.warp_group for op in ops], dtype=np.int32)
        rel = port.required_completion_relations(problem)
        self.rel = np.array([[self.index[a], self.index[b], d] for a, b, d in rel], dtype=np.int32).reshape(-1, 3)
        pairs = sorted({(u, d) for (_i, u), (_j, d) in port.carried_shared_lifetime_edges(problem)})
        self.car = np.array([[self.index[u], self.index[d]] for u, d in pairs], dtype=np.int32).reshape(-1, 2)
        owner, spaces, users = port.semantic_tables(problem)
        groups = []
        for value_id, space in spaces.items():
            if space != "register":
                continue
            component = set(users.get(value_id, ()))
            if value_id in owner:
                component.add(owner[value_id])
            if len(component) > 1:
                groups.append(sorted(self.index[item] for item in component))
        self.reg_off = np.array([0] + list(np.cumsum([len(g) for g in groups])), dtype=np.int32)
        self.reg_ops = np.array([k for g in groups for k in g] or [0], dtype=np.int32)
        resources = sorted(problem.resources, key=lambda item: item.id)
        res_index = {r.id: k for k, r in enumerate(resources)}
        self.cap = np.array([r.capacity for r in resources] or [0], dtype=np.int32)
        win_off, win_res, win_amt, win_dur = [0], [], [], []
        for op in ops:
            for w in op.resource_windows:
                win_res.append(res_index[w.resource_id])
                win_amt.append(w.amount)
                win_dur.append(w.duration)
            win_off.append(len(win_res))
        self.n_res = len(resources)
        self.win_off = np.array(win_off, dtype=np.int32)
        self.win_res = np.array(win_res or [0], dtype=np.int32)
        self.win_amt = np.array(win_amt or [0], dtype=np.int32)
        self.win_dur = np.array(win_dur or [0], dtype=np.int32)
        self._struct = _Problem(
            self.n, self.iterations, self.lanes,
            _ptr(self.issue), _ptr(self.latency), _ptr(self.wg),
            len(self.rel), _ptr(self.rel), len(self.car), _ptr(self.car),
            len(groups), _ptr(self.reg_off), _ptr(self.reg_ops),
            self.n_res, _ptr(self.cap), _ptr(self.win_off), _ptr(self.win_res), _ptr(self.win_amt), _ptr(self.win_dur),
        )

    # ------------------------------------------------------------------ structures
    def _frames(self, frames):
        """Flatten ``[(lanes, sync)]``; returns arrays plus per-frame class-1 flags."""
        lane_count, lane_base, lane_off, lane_ops = [], [], [], []
        sync_base, sync_count, sync_all = [], [], []
        malformed = []
        for lanes, sync in frames:
            try:
                lanes_c, sync_c, _ = port.construct(lanes, sync, [])
                malformed.append(False)
            except port.OracleFailure:
                lanes_c, sync_c = tuple(tuple(lane) for lane in lanes), list(sync)
                malformed.append(True)
            lane_count.append(len(lanes_c))
            lane_base.append(len(lane_off))
            for lane in lanes_c:
                lane_off.append(len(lane_ops))
                lane_ops.extend(self.index.get(op, -1) for op in lane)
            lane_off.append(len(lane_ops))
            sync_base.append(len(sync_all) // 3)
            sync_count.append(len(sync_c))
            for a, b, d in sync_c:
                sync_all.extend((self.index.get(a, -1), self.index.get(b, -1), min(int(d), 2**30)))
        as32 = lambda v: np.array(v or [0], dtype=np.int32)  # noqa: E731
        return (as32(lane_count), as32(lane_base), as32(lane_off), as32(lane_ops),
                as32(sync_base), as32(sync_count), as32(sync_all), np.array(malformed, dtype=bool))

    def new_memo(self, n_frames: int):
        """Per-frame answers of the reachability and acyclicity checks (-1: not asked yet)."""
        reach = np.full(max(1, n_frames) * max(1, len(self.rel) * self.iterations), -1, dtype=np.int8)
        return reach, np.full(max(1, n_frames), -1, dtype=np.int8)

    def _run(self, frame_arrays, frame_idx, pre, start, issue_end, completion, threads, memo=None):
        lib = _load()
        n = len(frame_idx)
        verdict = np.zeros(n, dtype=np.int32)
        if n == 0:
            return verdict
        lc, lb, lo, lops, sb, sc, sa, _ = frame_arrays
        memo_reach, memo_cycle = memo if memo is not None else self.new_memo(len(lc))
        M = self.n * self.iterations
        frame_idx = np.ascontiguousarray(frame_idx, dtype=np.int32)
        pre = np.ascontiguousarray(pre, dtype=np.int32)
        start = np.ascontiguousarray(start, dtype=np.int64).reshape(n, M)
        issue_end = np.ascontiguousarray(issue_end, dtype=np.int64).reshape(n, M)
        completion = np.ascontiguousarray(completion, dtype=np.int64).reshape(n, M)
        threads = max(1, threads or (os.cpu_count() or 1))
        bounds = np.linspace(0, n, min(threads * 4, n) + 1).astype(np.int64)

        def work(k: int) -> None:
            s, e = int(bounds[k]), int(bounds[k + 1])
            if e <= s:
                return
            lib.oracle_classify_batch(
                ctypes.byref(self._struct), 0, _ptr(lc), _ptr(lb), _ptr(lo), _ptr(lops), _ptr(sb), _ptr(sc), _ptr(sa),
                e - s, _ptr(frame_idx[s:e]), _ptr(pre[s:e]),
                _ptr(start[s:e], _i64p), _ptr(issue_end[s:e], _i64p), _ptr(completion[s:e], _i64p),
                _ptr(verdict[s:e]), memo_reach.ctypes.data, memo_cycle.ctypes.data,
            )

        with ThreadPoolExecutor(max_workers=threads) as pool:
            list(pool.map(work, range(len(bounds) - 1)))
        return verdict

    # ------------------------------------------------------------------ raw schedules
    def classify_raw(self, candidates, threads: int | None = None):
        """Classify raw ``(lanes, sync, rows)`` candidates -> (verdict, makespan, ii) arrays."""
        frames, frame_idx, pre = [], [], []
        n = len(candidates)
        M = self.n * self.iterations
        start = np.zeros((n, M), dtype=np.int64)
        issue_end = np.ones((n, M), dtype=np.int64)
        completion = np.ones((n, M), dtype=np.int64)
        makespan = np.zeros(n, dtype=np.int64)
        ii = np.zeros(n, dtype=np.int64)
        for k, (lanes, sync, rows) in enumerate(candidates):
            makespan[k], ii[k] = port.makespan_and_ii(self.problem, rows)
            frames.append((lanes, sync))
            frame_idx.append(k)
            try:
                _, _, times = port.construct(lanes, sync, rows)
            except port.OracleFailure:
                pre.append(1)
                continue
            expected = {(i, op) for i in range(self.iterations) for op in self.op_ids}
            if {(t[0], t[1]) for t in times} != expected:
                pre.append(7)
                continue
            pre.append(0)
            for i, op, s, e, c in times:
                r = i * self.n + self.index[op]
                start[k, r], issue_end[k, r], completion[k, r] = s, e, c
        verdict = self._run(self._frames(frames), np.array(frame_idx), np.array(pre), start, issue_end, completion, threads)
        return verdict, makespan, ii

    # ------------------------------------------------------------------ periodic batches
    def materialize(self, prologue: np.ndarray, offset: np.ndarray, ii: np.ndarray):
        """Rows of periodic candidates (solve.py:206-231), shape [n, I, N] int64."""
        prologue = np.asarray(prologue, dtype=np.int64)
        offset = np.asarray(offset, dtype=np.int64)
        ii = np.asarray(ii, dtype=np.int64)
        i = np.arange(self.iterations, dtype=np.int64)[None, :, None]
        start = offset[:, None, :] + i * ii[:, None, None]
        start[:, 0, :] = prologue
        issue_end = start + self.issue.astype(np.int64)[None, None, :]
        completion = start + self.latency.astype(np.int64)[None, None, :]
        return start, issue_end, completion

    def classify_periodic(self, prologue, offset, ii, frames, frame_idx, threads: int | None = None,
                          frame_arrays=None, memo=None):
        """Classify periodic candidates; ``prologue``/``offset`` are [n, N] absolute starts.

        Candidates are materialised in chunks of about 2^24 rows. ``frame_arrays`` and
        ``memo`` (see :meth:`prepare_frames`) may be passed to share the frames' answers
        between calls over the same frames.
        """
        prologue = np.asarray(prologue, dtype=np.int64)
        offset = np.asarray(offset, dtype=np.int64)
        ii = np.asarray(ii, dtype=np.int64)
        frame_idx = np.asarray(frame_idx, dtype=np.int32)
        if frame_arrays is None:
            frame_arrays, memo = self.prepare_frames(frames)
        n = prologue.shape[0]
        verdict = np.zeros(n, dtype=np.int32)
        makespan = np.zeros(n, dtype=np.int64)
        iiv = np.zeros(n, dtype=np.int64)
        chunk = max(1, (1 << 24) // max(1, self.n * self.iterations))
        for c0 in range(0, n, chunk):
            sl = slice(c0, min(n, c0 + chunk))
            start, issue_end, completion = self.materialize(prologue[sl], offset[sl], ii[sl])
            m = start.shape[0]
            makespan[sl] = completion.reshape(m, -1).max(axis=1)
            if self.iterations >= 3:
                iiv[sl] = start[:, 2, 0] - start[:, 1, 0]
            pre = np.where((start.reshape(m, -1) < 0).any(axis=1) | frame_arrays[-1][frame_idx[sl]], 1, 0)
            verdict[sl] = self._run(frame_arrays, frame_idx[sl], pre.astype(np.int32), start, issue_end, completion,
                                    threads, memo)
        return verdict, makespan, iiv

    def prepare_frames(self, frames):
        """Flattened frames and a fresh answer memo for :meth:`classify_periodic`."""
        arrays = self._frames(frames)
        return arrays, self.new_memo(len(frames))
