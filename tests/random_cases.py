"""Seeded random problems and raw schedules for parity tests (checked against the C oracle)."""

from __future__ import annotations

import numpy as np

from tilefoundry_b200 import pack_problem
from tilefoundry_b200.workloads import list_schedule_witness, random_dag_problem


def random_problem(seed: int):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(3, 100))
    lanes = int(rng.integers(1, 9))
    iterations = int(rng.choice([1, 2, 3, 4, 6, 9]))
    problem = random_dag_problem(
        n,
        layers=max(2, n // int(rng.integers(3, 10))),
        lanes=lanes,
        n_resources=int(rng.integers(0, 4)),
        iterations=iterations,
        seed=seed,
        latency=(4, 60),
        capacity=(2, 12),
        demand=(1, 4),
        carried=0.15,
        declared=float(rng.choice([1.0, 0.7, 0.0])),
    )
    packed = pack_problem(problem)
    return problem, packed, list_schedule_witness(packed, seed=seed)


def witness_rows(packed, witness, shift_body: np.ndarray | None = None):
    rows = []
    for i in range(packed.iterations):
        for k, op in enumerate(packed.op_ids):
            s = int(witness.prologue[k]) if i == 0 else int(witness.offset[k]) + i * witness.ii
            if shift_body is not None and i > 0:
                s += int(shift_body[i, k])
            rows.append([i, op, s, s + int(packed.issue[k]), s + int(packed.latency[k])])
    return rows


def raw_mutations(packed, witness, count: int, seed: int):
    """Raw ``(lanes, sync, rows)`` candidates around a valid witness (every verdict class)."""
    rng = np.random.default_rng(seed)
    out = []
    ops = list(packed.op_ids)
    for _ in range(count):
        lanes = [list(l) for l in witness.lanes]
        sync = [tuple(e) for e in witness.sync]
        rows = witness_rows(packed, witness)
        roll = rng.random()
        if roll < 0.08 and len(ops) > 1:  # swap two neighbours on a lane
            lane = max(lanes, key=len)
            if len(lane) >= 2:
                x = int(rng.integers(len(lane) - 1))
                lane[x], lane[x + 1] = lane[x + 1], lane[x]
        elif roll < 0.16 and sync:
            sync.pop(int(rng.integers(len(sync))))
        elif roll < 0.20:
            op = ops[int(rng.integers(len(ops)))]
            for lane in lanes:
                if op in lane:
                    lane.remove(op)
            lanes[int(rng.integers(len(lanes)))].append(op)
        elif roll < 0.23:
            lanes.append([])
        elif roll < 0.26:
            lanes[int(rng.integers(len(lanes)))].append("ghost")
        elif roll < 0.29:
            sync.append(("ghost", ops[0], 0))
        elif roll < 0.32:
            sync.append((ops[0], ops[-1], packed.iterations + int(rng.integers(0, 3))))
        roll = rng.random()
        if roll < 0.25:
            r = rows[int(rng.integers(len(rows)))]
            delta = int(rng.integers(-3, 4))
            r[2] += delta
            r[3] += delta
            r[4] += delta
        elif roll < 0.32:
            r = rows[int(rng.integers(len(rows)))]
            r[3 + int(rng.integers(2))] += int(rng.choice([-1, 1]))
        elif roll < 0.36:
            rows.pop(int(rng.integers(len(rows))))
        elif roll < 0.39:
            rows[int(rng.integers(len(rows)))][2] = -1
        elif roll < 0.55 and packed.iterations >= 2:  # tighten the body II
            cut = int(rng.integers(1, max(2, witness.ii // 2)))
            for r in rows:
                if r[0] > 0:
                    r[2] -= r[0] * cut
                    r[3] -= r[0] * cut
                    r[4] -= r[0] * cut
        out.append((lanes, sync, [tuple(r) for r in rows]))
    return out


def resource_heavy(seed: int, count: int):
    """A problem without dependencies whose candidates overlap iterations freely.

    Every operation reads only the external input, so there are no relations and sync is
    empty; lanes hold one or a few operations. Random prologue/offset starts and IIs make
    the resource capacity (class 20) the deciding check for most candidates, with the
    middle/boundary iterations of the periodic demand all exercised.
    """
    from tilefoundry_b200 import pack_problem
    from tilefoundry_b200.batch import FrameSet, PeriodicBatch

    rng = np.random.default_rng(seed)
    n = int(rng.integers(2, 16))
    problem = random_dag_problem(
        n, layers=1, lanes=n, n_resources=int(rng.integers(1, 4)), iterations=int(rng.choice([1, 2, 3, 5, 8, 13])),
        seed=seed, latency=(2, 40), capacity=(2, int(rng.integers(6, 40))), demand=(1, 4), windows_per_op=(1, 3),
        carried=0.0, declared=0.0,
    )
    packed = pack_problem(problem)
    frames = FrameSet(packed)
    frame = frames.add([[op] for op in packed.op_ids], [])  # one operation per lane
    span = int(packed.latency.max()) * 3
    issue = packed.issue.astype(np.int64)
    ii = rng.integers(int(issue.max()), span, size=count)
    prologue = rng.integers(0, span, size=(count, n))
    slack = np.maximum(ii[:, None] - issue[None, :], 0)
    offset = prologue + (rng.random((count, n)) * (slack + 1)).astype(np.int64)  # wrap edges hold
    batch = PeriodicBatch.from_starts(prologue, offset, ii, np.full(count, frame))
    return problem, packed, frames, batch


def resource_wide(seed: int, count: int, n_ops: int, n_resources: int, iterations: int = 4, lanes: int = 8):
    """Many operations on few resources: lanes of back-to-back operations, no dependencies.

    Each candidate draws its own gaps between the operations of a lane (prologue and body
    separately) and an II above its lane span for 85% of the batch, so the lane order
    holds for most candidates and the capacity check (class 20) decides them; each
    capacity is the median peak demand of a sample. With ``n_ops`` above 256 the
    global-read kernel runs, and a resource with more than 256 windows takes the
    one-thread-per-candidate path.
    """
    from tilefoundry_b200.batch import FrameSet, PeriodicBatch

    rng = np.random.default_rng(seed)
    problem = random_dag_problem(
        n_ops, layers=1, lanes=lanes, n_resources=n_resources, iterations=iterations, seed=seed,
        latency=(30, 200), capacity=(8, 160), demand=(1, 4), windows_per_op=(1, 1), carried=0.0, declared=0.0,
    )
    packed = pack_problem(problem)
    frames = FrameSet(packed)
    lane_of = np.arange(n_ops) % lanes
    frame = frames.add([[op for k, op in enumerate(packed.op_ids) if lane_of[k] == l] for l in range(lanes)], [])
    issue = packed.issue.astype(np.int64)

    def lane_starts():  # back-to-back lanes with per-candidate gaps of 0..7 cycles
        gaps = issue[None, :] + rng.integers(0, 8, size=(count, n_ops))
        starts = np.zeros((count, n_ops), dtype=np.int64)
        ends = np.zeros(count, dtype=np.int64)
        for l in range(lanes):
            ks = np.flatnonzero(lane_of == l)
            run = np.cumsum(gaps[:, ks], axis=1)
            starts[:, ks] = run - gaps[:, ks]
            ends = np.maximum(ends, run[:, -1])
        return starts, ends

    prologue, span_p = lane_starts()
    offset, span_o = lane_starts()
    prologue += rng.integers(0, 50, size=(count, 1))
    offset += rng.integers(0, 50, size=(count, 1))
    span = np.maximum(span_p, span_o)
    ii = span + rng.integers(60, 200, size=count)
    short = rng.random(count) < 0.15
    ii[short] = (span[short] * rng.uniform(0.5, 1.0, size=int(short.sum()))).astype(np.int64) + 1
    # Capacity of each resource: the median peak demand of a sample of the candidates, so
    # that about half of the lane-valid candidates exceed it.
    import dataclasses

    caps = []
    for q in range(n_resources):
        peaks = []
        for c in np.flatnonzero(~short)[:64]:
            events: dict[int, int] = {}
            for k in range(n_ops):
                for w in range(packed.window_offsets[k], packed.window_offsets[k + 1]):
                    if packed.window_resource[w] != q:
                        continue
                    for i in range(iterations):
                        s = int(prologue[c, k]) if i == 0 else int(offset[c, k] + i * ii[c])
                        events[s] = events.get(s, 0) + int(packed.window_amount[w])
                        events[s + int(packed.window_duration[w])] = events.get(s + int(packed.window_duration[w]), 0) - int(packed.window_amount[w])
            level = peak = 0
            for t in sorted(events):
                level += events[t]
                peak = max(peak, level)
            peaks.append(peak)
        caps.append(max(1, int(np.median(peaks))))
    resources = tuple(dataclasses.replace(r, capacity=caps[q]) for q, r in enumerate(problem.resources))
    problem = dataclasses.replace(problem, resources=resources)
    packed = pack_problem(problem)
    frames = FrameSet(packed)
    frame = frames.add([[op for k, op in enumerate(packed.op_ids) if lane_of[k] == l] for l in range(lanes)], [])
    batch = PeriodicBatch.from_starts(prologue, offset, ii, np.full(count, frame))
    return problem, packed, frames, batch
