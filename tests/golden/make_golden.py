"""Generate the golden verdict fixtures from the reference verifier itself.

Run in a container where the reference TileFoundry sources are available:

    python tests/golden/make_golden.py --reference /root/reference

The reference package needs its distribution metadata; the script creates a
temporary ``tilefoundry-0.0.0.dist-info`` next to a copy-free path entry, so the
reference tree is only read. For every problem it writes

* ``<name>_problem.json``  — the closed problem (format ``tilefoundry_b200.closed_problem``),
* ``<name>_raw.json.gz``   — raw candidates ``(lanes, sync, rows)`` with verdicts,
* ``<name>_periodic.npz``  — compact periodic candidates with verdicts,

where each verdict is ``(class_id, makespan, ii)``: the class id of the first
check the reference's ``_verify_warpgroup_schedule`` (verify.py:203-322) fails
(1 when a record constructor in model.py:425-507 refuses the schedule, 0 when
it verifies), the max completion (api.py:29-33) and ``start(2, first) -
start(1, first)`` for loops of three or more iterations (verify.py:261-262).

Problems: the repository's MLA decode example (examples/mla-schedule), and the
small problems of tests/schedule/test_warpgroup_schedule.py (`_program`
:76-119 with its hardware :122-145, `_periodic_resource_problem` :291-324 and
the shared-init problem :383-429) plus a variant of `_program` whose operations
leave their warp group undeclared.
"""

from __future__ import annotations

import argparse
import gzip
import json
import multiprocessing
import os
import random
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SEED = 20261201

PATTERNS = [
    ("schedule lane count does not match", 2),
    ("schedule repeats an operation across lanes", 3),
    ("schedule lane coverage differs", 4),
    ("expected warp_group", 5),
    ("schedule contains duplicate timed instances", 6),
    ("schedule time coverage differs", 7),
    ("wrong duration: issue duration", 8),
    ("wrong duration: completion latency", 9),
    ("periodic initiation interval must be positive", 10),
    ("periodic initiation interval differs", 11),
    ("lane order", 12),
    ("sync edge names an unknown operation", 13),
    ("sync edge has no finite instance", 14),
    ("sync inequality", 15),
    ("crosses warpgroup lanes", 16),
    ("has no lane/sync path", 18),
    ("completion relation", 17),
    ("carried shared lifetime", 19),
    ("exceeds capacity at time", 20),
    ("contains a cycle", 21),
]

REF = None  # module namespace filled by _import_reference


def _import_reference(root: Path) -> None:
    global REF
    meta = Path(tempfile.mkdtemp(prefix="tf_meta_"))
    info = meta / "tilefoundry-0.0.0.dist-info"
    info.mkdir()
    (info / "METADATA").write_text("Metadata-Version: 2.1\nName: tilefoundry\nVersion: 0.0.0\n")
    sys.path[:0] = [str(meta), str(root / "src")]
    import tilefoundry.schedule.warpgroup as wg
    from tilefoundry.schedule.warpgroup import build, verify

    class NS:
        pass

    REF = NS()
    REF.wg = wg
    REF.build = build.build_warpgroup_problem
    REF.verify = verify._verify_warpgroup_schedule


def reference_class(problem, lanes, sync, rows) -> int:
    wg = REF.wg
    try:
        schedule = wg.WarpgroupSchedule(
            wg.SCHEDULE_FORMAT,
            tuple(wg.WarpgroupLane(tuple(lane)) for lane in lanes),
            tuple(wg.SynchronizationEdge(a, b, d) for a, b, d in sync),
            tuple(wg.TimedOperation(*row) for row in rows),
        )
    except wg.WarpgroupValidationError:
        return 1
    try:
        REF.verify(problem, schedule)
    except wg.WarpgroupVerificationError as error:
        text = str(error)
        for pattern, class_id in PATTERNS:
            if pattern in text:
                return class_id
        raise RuntimeError(f"unmapped verifier message: {text}")
    return 0


def makespan_ii(problem, rows) -> tuple[int, int]:
    makespan = max((r[4] for r in rows), default=0)
    ii = 0
    if problem.loop.iterations >= 3:
        first = min(op.id for op in problem.loop.ops)
        starts = {(r[0], r[1]): r[2] for r in rows}
        if (2, first) in starts and (1, first) in starts:
            ii = starts[(2, first)] - starts[(1, first)]
    return makespan, ii


def materialize(problem, prologue, offset, ii):
    ops = sorted(problem.loop.ops, key=lambda o: o.id)
    rows = []
    for i in range(problem.loop.iterations):
        for k, op in enumerate(ops):
            s = int(prologue[k]) if i == 0 else int(offset[k]) + i * int(ii)
            rows.append((i, op.id, s, s + op.issue_duration, s + op.completion_latency))
    return rows


def problem_doc(problem) -> str:
    """Closed-problem document of a reference WarpgroupProblem."""
    from tilefoundry.schedule.warpgroup.expression import value_references

    doc = {
        "format": "tilefoundry_b200.closed_problem",
        "time_unit": problem.time_unit,
        "warp_groups": problem.warp_groups,
        "resources": [{"id": r.id, "capacity": r.capacity} for r in problem.resources],
        "types": [{"id": t.id, "space": t.space.value} for t in problem.types],
        "inputs": [{"id": i.id, "type_id": i.type_id} for i in problem.inputs],
        "loop": {
            "index": problem.loop.index,
            "iterations": problem.loop.iterations,
            "iter_args": [{"id": a.id, "yield": a.yield_value.id} for a in problem.loop.iter_args],
            "ops": [
                {
                    "id": op.id,
                    "warp_group": op.warp_group,
                    "issue_duration": op.issue_duration,
                    "completion_latency": op.completion_latency,
                    "resource_windows": [[w.resource_id, w.amount, w.duration] for w in op.resource_windows],
                    "outputs": [
                        {"id": o.id, "type_id": o.type_id, "uses": list(value_references(o.expression))}
                        for o in op.outputs
                    ],
                }
                for op in problem.loop.ops
            ],
        },
    }
    return json.dumps(doc, sort_keys=True, separators=(",", ":"))


# ----------------------------------------------------------------------------- problems


def small_problems():
    """The reference test-suite problems, rebuilt through the reference's own records."""
    wg = REF.wg
    T = wg.TensorType
    out = {}

    def tiny_program(iterations: int, declared: bool):
        types = (
            T("source", (iterations, 1), wg.DType.FP32, wg.MemorySpace.GLOBAL),
            T("shared", (1,), wg.DType.FP32, wg.MemorySpace.SHARED),
            T("value", (1,), wg.DType.FP32, wg.MemorySpace.REGISTER),
        )
        ops = (
            wg.ProgramOperation(
                "load",
                (wg.OperationOutput("%shared", "shared", wg.CopyExpression(
                    wg.IndexExpression(wg.ValueRef("%source"), (wg.LoopIndexRef("%iteration"),)))),),
                0 if declared else None,
            ),
            wg.ProgramOperation(
                "compute",
                (wg.OperationOutput("%result", "value",
                                    wg.ElementwiseExpression(wg.ElementwiseOperator.EXP, (wg.ValueRef("%shared"),))),),
                1 if declared else None,
            ),
            wg.ProgramOperation(
                "finish",
                (wg.OperationOutput("%final", "value",
                                    wg.ElementwiseExpression(wg.ElementwiseOperator.ADD,
                                                             (wg.ValueRef("%result"), wg.ScalarLiteral(1.0)))),),
                1 if declared else None,
            ),
            wg.ProgramOperation(
                "independent", (wg.OperationOutput("%independent", "value", wg.ScalarLiteral(1.0)),),
                2 if declared else None,
            ),
        )
        return wg.WarpgroupProgram(
            wg.PROGRAM_FORMAT, 4, types, (wg.ProgramInput("%source", "source"),),
            wg.ProgramLoop("%iteration", iterations, (), ops),
        )

    def tiny_hardware(program, capacity: int):
        costs = {}
        for op in program.loop.ops:
            sig = wg.operation_signature(program, op)
            if op.id == "load":
                cost = wg.OperationCost(1, 3, ())
            elif op.id == "compute":
                cost = wg.OperationCost(1, 2, (wg.ResourceWindow("engine", 1, 2),))
            elif op.id == "finish":
                cost = wg.OperationCost(2, 2, ())
            else:
                cost = wg.OperationCost(1, 1, (wg.ResourceWindow("engine", 1, 1),))
            costs[sig] = cost
        entries = tuple(wg.OperationCostEntry(s, c) for s, c in costs.items())
        return wg.WarpgroupHardware(wg.HARDWARE_FORMAT, "cycle", (wg.ResourceCapacity("engine", capacity),), entries)

    prog = tiny_program(3, True)
    out["tiny"] = REF.build(prog, tiny_hardware(prog, 1))
    prog = tiny_program(4, False)
    out["tiny_free"] = REF.build(prog, tiny_hardware(prog, 2))

    value_type = T("result", (1,), wg.DType.FP32, wg.MemorySpace.REGISTER)
    for capacity, window in ((1, 2), (2, 2), (4, 5), (5, 5)):
        out[f"resource_c{capacity}_w{window}"] = wg.model.WarpgroupProblem(
            "cycle", 2, (wg.ResourceCapacity("engine", capacity),), (value_type,), (),
            wg.model.ProblemLoop("%iteration", 3, (), (
                wg.model.ProblemOperation("early", (wg.OperationOutput("%early", "result", wg.ScalarLiteral(1.0)),),
                                          0, 1, window, (wg.ResourceWindow("engine", 1, window),)),
                wg.model.ProblemOperation("late", (wg.OperationOutput("%late", "result", wg.ScalarLiteral(2.0)),),
                                          1, 1, window + 1, (wg.ResourceWindow("engine", 1, window),)),
            )),
        )

    for iterations in (2, 4):
        types = (
            T("source", (iterations, 1), wg.DType.FP32, wg.MemorySpace.GLOBAL),
            T("shared", (1,), wg.DType.FP32, wg.MemorySpace.SHARED),
            T("result", (1,), wg.DType.FP32, wg.MemorySpace.REGISTER),
        )
        out[f"shared_init_i{iterations}"] = wg.model.WarpgroupProblem(
            "cycle", 2, (), types,
            (wg.ProgramInput("%source", "source"), wg.ProgramInput("%initial", "shared")),
            wg.model.ProblemLoop("%iteration", iterations,
                                 (wg.LoopIterArg("%carry", wg.ValueRef("%initial"), wg.ValueRef("%shared")),), (
                wg.model.ProblemOperation("publish", (wg.OperationOutput("%shared", "shared", wg.CopyExpression(
                    wg.IndexExpression(wg.ValueRef("%source"), (wg.LoopIndexRef("%iteration"),)))),), 0, 1, 1, ()),
                wg.model.ProblemOperation("consume", (wg.OperationOutput(
                    "%result", "result", wg.CopyExpression(wg.ValueRef("%carry"))),), 1, 4, 4, ()),
            )),
        )
    return out


# ----------------------------------------------------------------------------- candidates


def random_raw_candidate(problem, rng: random.Random):
    """One random schedule touching every verdict class with useful probability."""
    ops = sorted(op.id for op in problem.loop.ops)
    by_id = {op.id: op for op in problem.loop.ops}
    L, I = problem.warp_groups, problem.loop.iterations
    # lanes
    lanes = [[] for _ in range(L)]
    for op in ops:
        declared = by_id[op].warp_group
        lane = declared if (declared is not None and rng.random() < 0.9) else rng.randrange(L)
        lanes[lane].append(op)
    for lane in lanes:
        rng.shuffle(lane) if rng.random() < 0.3 else None
    roll = rng.random()
    if roll < 0.02:
        lanes.append([])
    elif roll < 0.04 and len(lanes) > 1:
        lanes.pop()
    elif roll < 0.06:
        lanes[rng.randrange(len(lanes))].append("ghost")
    elif roll < 0.08:
        victim = rng.choice(ops)
        for lane in lanes:
            if victim in lane:
                lane.remove(victim)
    elif roll < 0.09:
        lanes[0].append(lanes[0][0] if lanes[0] else ops[0])
    # sync: a subset of the required relations plus noise
    from tilefoundry.schedule.warpgroup.verify import _required_completion_relations

    required = [(r.after, r.before, r.distance) for r in _required_completion_relations(problem)]
    sync = [edge for edge in required if rng.random() < 0.8]
    if rng.random() < 0.3:
        a, b = rng.choice(ops), rng.choice(ops)
        sync.append((a, b, rng.choice([0, 1, 2, I, I + 1])))
    if rng.random() < 0.03:
        sync.append(("ghost", rng.choice(ops), 0))
    if rng.random() < 0.02 and sync:
        sync.append(sync[0])
    # times: periodic most of the time, else raw noise
    base = {op: rng.randrange(0, 6 * len(ops)) for op in ops}
    ii = rng.randrange(-1, 4 * len(ops) + 4)
    rows = []
    for i in range(I):
        for op in ops:
            o = by_id[op]
            s = base[op] if i == 0 else base[op] + 2 + i * ii
            rows.append([i, op, s, s + o.issue_duration, s + o.completion_latency])
    roll = rng.random()
    if roll < 0.05:
        r = rng.choice(rows)
        r[3] += rng.choice([-1, 1])
    elif roll < 0.10:
        r = rng.choice(rows)
        r[4] += rng.choice([-1, 1])
    elif roll < 0.15:
        r = rng.choice(rows)
        r[2] -= 1
        r[3] -= 1
        r[4] -= 1
    elif roll < 0.18:
        rows.pop(rng.randrange(len(rows)))
    elif roll < 0.20:
        rows.append([I, ops[0], 0, by_id[ops[0]].issue_duration, by_id[ops[0]].completion_latency])
    elif roll < 0.22:
        rows.append(list(rows[0]))
    elif roll < 0.25:
        r = rng.choice(rows)
        r[2] = -1
    rows = [tuple(r) for r in rows]
    return [list(lane) for lane in lanes], [list(e) for e in sync], [list(r) for r in rows]


def search_valid_periodic(problem, frame, rng: random.Random, tries: int = 400):
    """A few (prologue, offset, ii) that verify for this frame, by random search."""
    ops = sorted(problem.loop.ops, key=lambda o: o.id)
    found = []
    for _ in range(tries):
        span = 4 * sum(o.completion_latency for o in ops)
        p = [rng.randrange(0, span) for _ in ops]
        o = [rng.randrange(0, span) for _ in ops]
        ii = rng.randrange(1, span + 2)
        rows = materialize(problem, p, o, ii)
        if reference_class(problem, frame[0], frame[1], rows) == 0:
            found.append((p, o, ii))
            if len(found) >= 4:
                break
    return found


def periodic_candidates_small(problem, rng: random.Random, count: int):
    """Periodic candidates over a handful of frames, around valid points when found."""
    ops = sorted(problem.loop.ops, key=lambda o: o.id)
    n = len(ops)
    frames = []
    for _ in range(6):
        lanes, sync, _ = random_raw_candidate(problem, rng)
        frames.append((lanes, sync))
    anchors = {k: search_valid_periodic(problem, frames[k], rng) for k in range(len(frames))}
    P, O, II, F = [], [], [], []
    for _ in range(count):
        k = rng.randrange(len(frames))
        if anchors[k] and rng.random() < 0.7:
            p, o, ii = rng.choice(anchors[k])
            p = [v + rng.choice([0, 0, 0, -1, 1, -2, 2]) for v in p]
            o = [v + rng.choice([0, 0, 0, -1, 1, -2, 2]) for v in o]
            ii = ii + rng.choice([0, 0, 0, -1, 1])
        else:
            span = 4 * sum(op.completion_latency for op in ops)
            p = [rng.randrange(-2, span) for _ in range(n)]
            o = [rng.randrange(-2, span) for _ in range(n)]
            ii = rng.randrange(-2, span)
        P.append(p)
        O.append(o)
        II.append(ii)
        F.append(k)
    return frames, np.array(P, dtype=np.int64), np.array(O, dtype=np.int64), np.array(II, dtype=np.int64), np.array(F)


# ----------------------------------------------------------------------------- MLA


def mla(root: Path):
    wg = REF.wg
    example = root / "examples" / "mla-schedule"
    program = wg.warpgroup_program_from_json((example / "program.json").read_text())
    hardware = wg.warpgroup_hardware_from_json((example / "hardware.json").read_text())
    schedule = wg.warpgroup_schedule_from_json((example / "schedule.json").read_text())
    problem = REF.build(program, hardware)
    return problem, schedule


def mla_periodic(problem, schedule, rng: np.random.Generator, count: int):
    """Seeded perturbations of the committed MLA schedule in compact periodic form."""
    ops = sorted(op.id for op in problem.loop.ops)
    index = {op: k for k, op in enumerate(ops)}
    times = {(t.iteration, t.operation_id): t.start for t in schedule.times}
    ii0 = times[(2, ops[0])] - times[(1, ops[0])]
    P0 = np.array([times[(0, op)] for op in ops], dtype=np.int64)
    O0 = np.array([times[(1, op)] - ii0 for op in ops], dtype=np.int64)
    lanes0 = [list(lane.operations) for lane in schedule.lanes]
    sync0 = [[e.after, e.before, e.distance] for e in schedule.sync]
    shared_ops = {op.id for op in problem.loop.ops
                  if any(o.type_id in {t.id for t in problem.types if t.space.value == "shared"} for o in op.outputs)}
    frames = [(lanes0, sync0)]
    P, O, II, F = [], [], [], []
    for _ in range(count):
        p, o, ii, f = P0.copy(), O0.copy(), ii0, 0
        kind = rng.random()
        if kind < 0.30:  # jitter a few operations
            for k in rng.choice(len(ops), size=rng.integers(1, 4), replace=False):
                p[k] += rng.integers(-64, 65)
                o[k] += rng.integers(-64, 65)
        elif kind < 0.45:  # move everything later (stays valid)
            shift = rng.integers(0, 400)
            p += shift
            o += shift + rng.integers(0, 64)
        elif kind < 0.55:  # one operation onto another warpgroup
            lanes = [list(l) for l in lanes0]
            op = ops[rng.integers(len(ops))]
            for lane in lanes:
                if op in lane:
                    lane.remove(op)
            target = rng.integers(len(lanes))
            lanes[target].insert(rng.integers(len(lanes[target]) + 1), op)
            frames.append((lanes, sync0))
            f = len(frames) - 1
        elif kind < 0.60:  # swap two shared-producing operations of one lane
            lanes = [list(l) for l in lanes0]
            lane = lanes[rng.integers(len(lanes))]
            cands = [k for k, op in enumerate(lane) if op in shared_ops] or list(range(len(lane)))
            if len(cands) >= 2:
                x, y = rng.choice(cands, size=2, replace=False)
                lane[x], lane[y] = lane[y], lane[x]
            frames.append((lanes, sync0))
            f = len(frames) - 1
        elif kind < 0.70:  # drop one sync edge
            drop = rng.integers(len(sync0))
            frames.append((lanes0, [e for j, e in enumerate(sync0) if j != drop]))
            f = len(frames) - 1
        elif kind < 0.78:  # change the initiation interval
            ii = ii0 + int(rng.integers(-40, 41))
            if rng.random() < 0.1:
                ii = -ii0 if rng.random() < 0.5 else 0
        elif kind < 0.82:  # a negative start
            p[rng.integers(len(ops))] = -int(rng.integers(1, 50))
        else:  # unchanged witness
            pass
        P.append(p)
        O.append(o)
        II.append(ii)
        F.append(f)
    return frames, np.array(P), np.array(O), np.array(II, dtype=np.int64), np.array(F)


def mla_raw_cases(problem, schedule, rng: random.Random):
    ops = sorted(op.id for op in problem.loop.ops)
    lanes0 = [list(lane.operations) for lane in schedule.lanes]
    sync0 = [[e.after, e.before, e.distance] for e in schedule.sync]
    rows0 = [[t.iteration, t.operation_id, t.start, t.issue_end, t.completion] for t in schedule.times]
    cases = [(lanes0, sync0, rows0)]

    def variant(lanes=None, sync=None, rows=None):
        cases.append((lanes if lanes is not None else [list(l) for l in lanes0],
                      sync if sync is not None else [list(e) for e in sync0],
                      rows if rows is not None else [list(r) for r in rows0]))

    variant(lanes=[list(l) for l in lanes0] + [[]])
    variant(lanes=[lanes0[0] + ["ghost_op"], lanes0[1], lanes0[2]])
    variant(lanes=[lanes0[0][1:], lanes0[1], lanes0[2]])
    variant(lanes=[lanes0[0] + [lanes0[1][0]], lanes0[1][1:], lanes0[2]])
    variant(rows=rows0[:-1])
    for k in range(6):
        rows = [list(r) for r in rows0]
        r = rows[rng.randrange(len(rows))]
        which = k % 3
        if which == 0:
            r[3] += 1
        elif which == 1:
            r[4] += 1
        else:
            r[2] += 1
            r[3] += 1
            r[4] += 1
        variant(rows=rows)
    variant(sync=sync0 + [["ghost_op", ops[0], 0]])
    variant(sync=sync0 + [[ops[0], ops[1], problem.loop.iterations]])
    variant(sync=sync0 + [[ops[0], ops[1], 5]])
    variant(sync=sync0 + [sync0[0]])
    rows = [list(r) for r in rows0]
    rows[5][2] = -3
    variant(rows=rows)
    for drop in range(0, len(sync0), 5):
        variant(sync=[e for j, e in enumerate(sync0) if j != drop])
    return cases


# ----------------------------------------------------------------------------- main


def _label(args):
    problem_key, lanes, sync, rows = args
    problem = _PROBLEMS[problem_key]
    rows_t = [tuple(r) for r in rows]
    cls = reference_class(problem, lanes, [tuple(e) for e in sync], rows_t)
    return (cls, *makespan_ii(problem, rows_t))


_PROBLEMS: dict = {}


def _init_worker(root: str) -> None:
    _import_reference(Path(root))
    _PROBLEMS.update(small_problems())
    _PROBLEMS["mla"] = mla(Path(root))[0]


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default="/root/reference")
    parser.add_argument("--mla-periodic", type=int, default=384)
    parser.add_argument("--small-raw", type=int, default=600)
    parser.add_argument("--small-periodic", type=int, default=600)
    parser.add_argument("--workers", type=int, default=os.cpu_count() or 1)
    args = parser.parse_args()
    root = Path(args.reference)
    _init_worker(str(root))
    rng = random.Random(SEED)
    nrng = np.random.default_rng(SEED)
    problem, schedule = mla(root)
    with multiprocessing.get_context("fork").Pool(args.workers, initializer=_init_worker, initargs=(str(root),)) as pool:
        jobs = {"mla": (problem, mla_raw_cases(problem, schedule, rng))}
        for name, prob in small_problems().items():
            jobs[name] = (prob, [random_raw_candidate(prob, rng) for _ in range(args.small_raw)])
        for name, (prob, cases) in jobs.items():
            (HERE / f"{name}_problem.json").write_text(problem_doc(prob))
            labels = pool.map(_label, [(name, *case) for case in cases], chunksize=4)
            payload = {"problem": name, "candidates": [list(case) for case in cases], "verdicts": [list(v) for v in labels]}
            with gzip.open(HERE / f"{name}_raw.json.gz", "wt", encoding="utf-8") as handle:
                handle.write(json.dumps(payload, separators=(",", ":")))
            hist = np.bincount([v[0] for v in labels], minlength=22)
            print(name, "raw", len(cases), "classes", {k: int(c) for k, c in enumerate(hist) if c})

        periodic = {"mla": (problem, *mla_periodic(problem, schedule, nrng, args.mla_periodic))}
        for name, prob in small_problems().items():
            periodic[name] = (prob, *periodic_candidates_small(prob, rng, args.small_periodic))
        for name, (prob, frames, P, O, II, F) in periodic.items():
            work = [(name, frames[f][0], frames[f][1], materialize(prob, P[k], O[k], II[k])) for k, f in enumerate(F)]
            labels = np.array(pool.map(_label, work, chunksize=2), dtype=np.int64)
            np.savez_compressed(
                HERE / f"{name}_periodic.npz",
                frames=np.array(json.dumps(frames)), prologue=P, offset=O, ii=II, frame=F,
                verdict=labels[:, 0], makespan=labels[:, 1], iiv=labels[:, 2],
            )
            hist = np.bincount(labels[:, 0], minlength=22)
            print(name, "periodic", len(F), "frames", len(frames), "classes",
                  {k: int(c) for k, c in enumerate(hist) if c})


if __name__ == "__main__":
    main()
