"""GPU canonical synchronization export (drop-in for sync.py:21-62) against the oracle.

The committed MLA schedule is the reference's own export, so re-exporting its lanes and
times must keep exactly its sync edges; random layered-DAG witnesses are compared with
``oracle/verify_port.py``'s restatement of the export, including schedules whose complete
candidate set does not verify.
"""

from __future__ import annotations

import numpy as np
import pytest

from golden_data import problem_text, raw_cases
from oracle import verify_port as port
from oracle.problem_doc import load_problem
from random_cases import witness_rows
from tilefoundry_b200 import (
    TimedOperation,
    WarpgroupLane,
    WarpgroupSolveResult,
    WarpgroupVerificationError,
    export_warpgroup_schedule,
    export_warpgroup_schedules,
    pack_problem,
    problem_from_json,
    problem_to_json,
)
from tilefoundry_b200.workloads import list_schedule_witness, random_dag_problem

pytestmark = pytest.mark.gpu


def _result(lanes, rows):
    return WarpgroupSolveResult(
        "OPTIMAL",
        tuple(WarpgroupLane(tuple(lane)) for lane in lanes),
        tuple(TimedOperation(*row) for row in rows),
    )


def test_export_reproduces_the_reference_exported_mla_sync():
    problem = problem_from_json(problem_text("mla"))
    lanes, sync, rows = raw_cases("mla")[0][0]
    schedule = export_warpgroup_schedule(problem, _result(lanes, rows))
    got = sorted((e.after, e.before, e.distance) for e in schedule.sync)
    assert got == sorted(tuple(e) for e in sync)
    assert len(got) == 48


def _small_problem(seed):
    rng = np.random.default_rng(seed)
    problem = random_dag_problem(
        int(rng.integers(4, 28)), layers=int(rng.integers(2, 6)), lanes=int(rng.integers(1, 5)), n_resources=0,
        iterations=int(rng.choice([1, 2, 3, 4])), seed=seed, latency=(2, 30), carried=0.2,
        declared=float(rng.choice([1.0, 0.0])),
    )
    return problem, pack_problem(problem)


@pytest.mark.parametrize("seed", range(12))
def test_export_matches_oracle_on_random_witnesses(seed):
    problem, packed = _small_problem(seed)
    witness = list_schedule_witness(packed, seed=seed)
    rows = witness_rows(packed, witness)
    rng = np.random.default_rng(seed + 100)
    results, expected = [], []
    oracle_problem = load_problem(problem_to_json(problem))
    for variant in range(6):
        lanes = [list(lane) for lane in witness.lanes]
        vrows = [list(r) for r in rows]
        if variant >= 3 and len(vrows) > 1:  # pull one instance earlier: the complete set may fail
            r = vrows[int(rng.integers(len(vrows)))]
            shift = min(int(r[2]), int(rng.integers(1, 40)))
            r[2] -= shift
            r[3] -= shift
            r[4] -= shift
        if variant % 3 == 2:  # another lane assignment of the same times
            longest = max(lanes, key=len)
            if len(longest) > 1 and len(lanes) > 1:
                op = longest.pop()
                min(lanes, key=len).append(op)
        vrows = [tuple(r) for r in vrows]
        if any(r[2] < 0 for r in vrows):
            continue
        results.append(_result(lanes, vrows))
        clanes, _csync, crows = port.construct(lanes, [], vrows)
        expected.append(port.export_sync(oracle_problem, clanes, crows))
    got = export_warpgroup_schedules(problem, results)
    assert any(status == "ok" for status, _ in expected)
    for found, (status, value) in zip(got, expected):
        if status == "ok":
            assert not isinstance(found, BaseException), found
            assert [(e.after, e.before, e.distance) for e in found.sync] == sorted(value)
        else:
            assert isinstance(found, BaseException)


def test_export_rejects_inexact_records_and_bad_lanes():
    problem = problem_from_json(problem_text("mla"))
    lanes, _sync, rows = raw_cases("mla")[0][0]
    result = _result(lanes, rows)
    with pytest.raises(WarpgroupVerificationError, match="exact WarpgroupSolveResult"):
        export_warpgroup_schedule(problem, (result.lanes, result.times))
    short = _result(lanes[:-1] + [[]], rows)
    with pytest.raises(WarpgroupVerificationError, match="do not exactly cover"):
        export_warpgroup_schedule(problem, short)
