"""Host-side logic: codecs, problem packing, frame/row packing, workloads, sharding (CPU only)."""

from __future__ import annotations

import os

import numpy as np
import pytest

from golden_data import PROBLEMS, problem_text, raw_cases
from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem
from tilefoundry_b200 import (
    SCHEDULE_FORMAT,
    SynchronizationEdge,
    TimedOperation,
    WarpgroupLane,
    WarpgroupSchedule,
    WarpgroupSerializationError,
    WarpgroupValidationError,
    pack_problem,
    problem_from_json,
    problem_to_json,
    schedule_from_json,
    schedule_to_json,
)
from tilefoundry_b200 import _lib
from tilefoundry_b200.batch import FrameSet, PeriodicBatch, pack_rows
from tilefoundry_b200.shard import shard_bounds
from tilefoundry_b200.workloads import absolute_starts, mla_perturbations, shared_producers, witness_from_rows


def mla():
    problem = problem_from_json(problem_text("mla"))
    cases, _ = raw_cases("mla")
    return problem, pack_problem(problem), cases[0]


@pytest.mark.parametrize("name", PROBLEMS)
def test_problem_document_round_trip(name):
    problem = problem_from_json(problem_text(name))
    assert problem_from_json(problem_to_json(problem)) == problem


@pytest.mark.parametrize("name", PROBLEMS)
def test_packed_tables_match_oracle_derivation(name):
    packed = pack_problem(problem_from_json(problem_text(name)))
    oracle = OracleProblem(load_problem(problem_text(name)))
    assert packed.op_ids == tuple(oracle.op_ids)
    assert np.array_equal(packed.issue, oracle.issue)
    assert np.array_equal(packed.latency, oracle.latency)
    assert np.array_equal(packed.warp_group, oracle.wg)
    assert np.array_equal(packed.relations, oracle.rel)
    assert np.array_equal(packed.carried, oracle.car)
    groups = lambda off, ops: sorted(tuple(ops[off[g]:off[g + 1]]) for g in range(len(off) - 1))  # noqa: E731
    assert groups(packed.register_offsets, packed.register_ops) == groups(oracle.reg_off, oracle.reg_ops)
    assert np.array_equal(packed.window_offsets, oracle.win_off)


def test_schedule_document_round_trip_and_strictness():
    _problem, _packed, (lanes, sync, rows) = mla()
    schedule = WarpgroupSchedule(
        SCHEDULE_FORMAT,
        tuple(WarpgroupLane(tuple(lane)) for lane in lanes),
        tuple(SynchronizationEdge(*edge) for edge in sync),
        tuple(TimedOperation(*row) for row in rows),
    )
    text = schedule_to_json(schedule)
    assert schedule_from_json(text) == schedule
    with pytest.raises(WarpgroupSerializationError):
        schedule_from_json(text.replace('"format"', '"fmt"'))
    with pytest.raises(WarpgroupSerializationError):
        schedule_from_json(text.replace(SCHEDULE_FORMAT, SCHEDULE_FORMAT + ".v2"))


def test_schedule_constructor_rules_match_reference():
    with pytest.raises(WarpgroupValidationError):
        TimedOperation(0, "a", -1, 1, 2)
    with pytest.raises(WarpgroupValidationError):
        TimedOperation(0, "a", 3, 3, 4)
    with pytest.raises(WarpgroupValidationError):
        SynchronizationEdge("a", "a", 0)
    with pytest.raises(WarpgroupValidationError):
        WarpgroupLane(("a", "a"))
    with pytest.raises(WarpgroupValidationError):
        WarpgroupSchedule(SCHEDULE_FORMAT, (WarpgroupLane(("a",)), WarpgroupLane(("a",))), (), ())


def test_frame_packing_flags_and_permutation():
    _problem, packed, (lanes, sync, _rows) = mla()
    frames = FrameSet(packed)
    base = frames.add(lanes, sync)
    assert frames.add(lanes, sync) == base
    arrays = frames.arrays()
    pos = arrays["lane_pos"][base]
    for lane_index, lane in enumerate(lanes):
        got = sorted((int(p) & 0xFFF, packed.op_ids[k]) for k, p in enumerate(pos) if int(p) >> 12 == lane_index)
        assert [op for _, op in got] == lane
    assert arrays["flags"][base] == 0
    ghost = frames.add([lanes[0] + ["ghost"], lanes[1], lanes[2]], sync)
    dup = frames.add([lanes[0] + [lanes[1][0]], lanes[1], lanes[2]], sync)
    bad_sync = frames.add(lanes, list(sync) + [(lanes[0][0], lanes[0][0], 0)])
    missing = frames.add([lanes[0][1:], lanes[1], lanes[2]], sync)
    arrays = frames.arrays()
    assert arrays["flags"][ghost] == _lib.TFV_FRAME_UNKNOWN_LANE_OP
    assert arrays["flags"][dup] & _lib.TFV_FRAME_MALFORMED
    assert arrays["flags"][bad_sync] & _lib.TFV_FRAME_MALFORMED
    assert (arrays["lane_pos"][missing] >> 12 == 15).sum() == 1
    assert arrays["sync_offsets"][-1] == arrays["sync_edges"].shape[0]


def test_rows_packing_flags_coverage_and_overrides():
    problem, packed, (lanes, sync, rows) = mla()
    frames = FrameSet(packed)
    missing = rows[:-1]
    extra = list(rows) + [(99, packed.op_ids[0], 0, 1, 1000000)]
    negative = [(r[0], r[1], -1, r[3], r[4]) if k == 3 else r for k, r in enumerate(rows)]
    batch = pack_rows(packed, frames, [(lanes, sync, rows), (lanes, sync, missing), (lanes, sync, extra), (lanes, sync, negative)])
    assert list(batch.row_flags) == [0, _lib.TFV_ROWS_COVERAGE, _lib.TFV_ROWS_COVERAGE, _lib.TFV_ROWS_MALFORMED]
    assert batch.override_makespan[2] == 1000000
    assert batch.start.shape == (4, packed.iterations, packed.n_ops)
    assert batch.start[1].max() == batch.start[0].max()


def test_periodic_batch_from_starts_round_trip_and_range():
    rng = np.random.default_rng(3)
    prologue = rng.integers(0, 50000, size=(7, 5))
    offset = prologue + rng.integers(0, 100, size=(7, 5))
    batch = PeriodicBatch.from_starts(prologue, offset, np.full(7, 10), np.zeros(7))
    p, o = absolute_starts(batch)
    assert np.array_equal(p, prologue) and np.array_equal(o, offset)
    with pytest.raises(ValueError):
        PeriodicBatch.from_starts(np.array([[0], [100000]]), np.array([[0], [0]]), [1, 1], [0, 0])


def test_mla_workload_mix_is_about_half_invalid():
    problem, packed, case = mla()
    witness = witness_from_rows(packed, *case)
    assert witness.ii == 3806
    frames, batch, kind = mla_perturbations(packed, witness, 3000, seed=11, producers=shared_producers(problem))
    oracle = OracleProblem(load_problem(problem_text("mla")))
    p, o = absolute_starts(batch)
    verdict, makespan, ii = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert 0.25 < (verdict == 0).mean() < 0.65
    assert {0, 5, 12, 15, 18} <= set(np.unique(verdict).tolist())
    assert (ii == batch.ii).all()


def test_shard_bounds_cover_exactly():
    for n in (0, 1, 7, 1000):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def _gather_worker(rank: int, world: int, port: int, queue) -> None:
    import torch
    import torch.distributed as dist

    from tilefoundry_b200.shard import gather_results, shard_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n = 11
    lo, hi = shard_bounds(n, rank, world)
    values = torch.arange(lo, hi, dtype=torch.int32)
    full = gather_results((values, values * 2, values * 3), n)
    if rank == 0:
        queue.put(full.tolist())
    dist.destroy_process_group()


def test_gather_results_two_gloo_ranks():
    import multiprocessing as mp
    import socket

    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, queue)) for r in range(2)]
    for proc in procs:
        proc.start()
    full = queue.get(timeout=120)
    for proc in procs:
        proc.join(timeout=60)
        assert proc.exitcode == 0
    assert full[0] == list(range(11))
    assert full[2] == [3 * v for v in range(11)]


def test_ii_lower_bound_and_sweep():
    """solve.py:186-204, 261-264 from the problem records: max issue duration and, per
    resource, ceil(sum of duration * amount / capacity)."""
    from tilefoundry_b200 import pack_problem
    from tilefoundry_b200.workloads import ii_lower_bound, ii_sweep, random_dag_problem

    for seed in range(6):
        problem = random_dag_problem(40, layers=4, lanes=4, n_resources=3, iterations=4, seed=seed,
                                     latency=(2, 300), capacity=(2, 9))
        held: dict[str, int] = {}
        for op in problem.loop.ops:
            for w in op.resource_windows:
                held[w.resource_id] = held.get(w.resource_id, 0) + w.duration * w.amount
        capacity = {r.id: r.capacity for r in problem.resources}
        want = max([max(op.issue_duration for op in problem.loop.ops)] +
                   [-(-total // capacity[rid]) for rid, total in held.items()])
        assert ii_lower_bound(pack_problem(problem)) == want
    values = ii_sweep(100, 16)
    assert values[0] == 100 and values[-1] == 200 and len(values) == 16 and np.all(np.diff(values) > 0)
    assert ii_sweep(7, 1).tolist() == [7]


def test_closed_problem_is_built_once_per_document_pair():
    from tilefoundry_b200.verify import closed_problem

    calls = []

    def build(program, hardware):
        calls.append((program, hardware))
        return ("problem", len(calls))

    from dataclasses import dataclass

    @dataclass(frozen=True)
    class Document:
        name: str

    program, hardware, other = Document("program"), Document("hardware"), Document("other")
    first = closed_problem(program, hardware, build)
    assert closed_problem(program, hardware, build) is first
    assert closed_problem(program, other, build) is not first
    assert len(calls) == 2


def test_closed_problem_rebuilds_for_mutable_cost_libraries():
    """A cost library that is not an immutable record may change between calls (the
    reference accepts any object with lookup() and resources, cost.py:166-175): it is closed
    again on every call, as the reference does (verify.py:325-331)."""
    from dataclasses import dataclass

    from tilefoundry_b200.verify import closed_problem

    @dataclass(frozen=True)
    class Program:
        name: str

    class Library:  # a stateful provider
        resources = ()

        def lookup(self, signature):
            return None

    calls = []

    def build(program, hardware):
        calls.append(1)
        return ("problem", len(calls))

    program, library = Program("p"), Library()
    assert closed_problem(program, library, build) == ("problem", 1)
    assert closed_problem(program, library, build) == ("problem", 2)


def _packed_worker(rank, world, port, queue):
    import os

    import torch
    import torch.distributed as dist

    from tilefoundry_b200.shard import gather_packed, pack_results, shard_bounds, unpack_results

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = shard_bounds(13, rank, world)
    idx = torch.arange(lo, hi, dtype=torch.int32)
    verdict = (idx % 26) - 4                     # every class, -4 .. 21
    makespan = idx * 1000003 + 7
    packed = pack_results(verdict, makespan)
    v, m = unpack_results(packed, hi - lo)
    assert torch.equal(v, verdict) and torch.equal(m, makespan)
    full = gather_packed(packed, 13)
    if rank == 0:
        queue.put((full[0].tolist(), full[1].tolist()))
    dist.destroy_process_group()


def test_gather_packed_two_gloo_ranks():
    import multiprocessing as mp
    import socket

    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_packed_worker, args=(r, 2, port, queue)) for r in range(2)]
    for proc in procs:
        proc.start()
    verdict, makespan = queue.get(timeout=120)
    for proc in procs:
        proc.join(timeout=60)
        assert proc.exitcode == 0
    assert verdict == [(i % 26) - 4 for i in range(13)]
    assert makespan == [i * 1000003 + 7 for i in range(13)]


def test_periodic_groups_cover_outliers_exactly():
    """Candidates whose starts leave the int16 range of the batch base are split off into
    batches of their own; every candidate lands in one batch and its starts are exact."""
    from tilefoundry_b200.batch import periodic_groups

    rng = np.random.default_rng(4)
    n, N = 5000, 7
    prologue = rng.integers(0, 3000, size=(n, N)).astype(np.int64)
    offset = prologue + rng.integers(0, 500, size=(n, N))
    out = rng.random(n) < 0.01
    prologue[out, rng.integers(0, N, size=int(out.sum()))] += rng.choice([-1, 1], size=int(out.sum())) * 100000
    offset[out] += 150000
    ii = rng.integers(1, 9000, size=n)
    frame = rng.integers(0, 3, size=n)
    groups = periodic_groups(prologue, offset, ii, frame)
    seen = np.concatenate([take for take, _ in groups])
    assert sorted(seen.tolist()) == list(range(n))
    assert len(groups) >= 2 and groups[0][0].size > 0.95 * n
    for take, batch in groups:
        assert np.array_equal(batch.base_prologue[None, :] + batch.prologue_delta.T.astype(np.int64), prologue[take])
        assert np.array_equal(batch.base_offset[None, :] + batch.offset_delta.T.astype(np.int64), offset[take])
        assert np.array_equal(batch.ii, ii[take]) and np.array_equal(batch.frame, frame[take])
