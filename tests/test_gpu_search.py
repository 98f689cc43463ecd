"""The GPU-oracle neighbourhood search: every accepted schedule verifies (oracle-checked),
the (II, makespan) objective never gets worse, and the result exports and round-trips."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem
from tilefoundry_b200 import (
    _verify_warpgroup_schedule,
    export_warpgroup_schedule,
    pack_problem,
    problem_to_json,
    schedule_from_json,
    schedule_to_json,
)
from tilefoundry_b200.batch import FrameSet, PeriodicBatch
from tilefoundry_b200.search import improve_periodic
from tilefoundry_b200.workloads import absolute_starts, gemm_mainloop_problem, list_schedule_witness, random_dag_problem

pytestmark = pytest.mark.gpu


def _oracle_verdict(problem, packed, witness):
    frames = FrameSet(packed)
    f = frames.add(witness.lanes, witness.sync)
    batch = PeriodicBatch.from_starts(witness.prologue[None, :], witness.offset[None, :], np.array([witness.ii]),
                                      np.array([f]))
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    p, o = absolute_starts(batch)
    v, m, i = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    return int(v[0]), int(m[0]), int(i[0])


@pytest.mark.parametrize("which", ["dag", "gemm"])
def test_search_improves_and_every_result_verifies(which):
    if which == "dag":
        problem = random_dag_problem(24, layers=4, lanes=3, n_resources=2, iterations=6, seed=3, latency=(4, 80),
                                     capacity=(6, 20))
    else:
        problem = gemm_mainloop_problem()
    packed = pack_problem(problem)
    witness = list_schedule_witness(packed, seed=1)
    v0, m0, _ = _oracle_verdict(problem, packed, witness)
    assert v0 == 0
    result = improve_periodic(problem, witness, rounds=8, batch=1 << 14, seed=7)
    v, m, ii = _oracle_verdict(problem, packed, result.witness)
    assert v == 0 and m == result.makespan
    assert (result.ii, result.makespan) <= (witness.ii, m0)
    assert result.accepted > 0  # a list-scheduled witness with II = span leaves room
    keys = [(a, b) for a, b in result.history]
    assert keys == sorted(keys, reverse=True)
    # the improved schedule exports (GPU sync export), round-trips as JSON and verifies
    exported = export_warpgroup_schedule(problem, result.solve_result(packed))
    again = schedule_from_json(schedule_to_json(exported))
    _verify_warpgroup_schedule(problem, again)
