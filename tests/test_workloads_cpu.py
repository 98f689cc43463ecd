"""The body generators (workloads.body_batch) on the CPU, checked by the oracle: the
calibrated GEMM and FlashAttention batches hold verified schedules and capacity failures
(class 20) beside the lane, sync and relation failures, every delta fits the batch's int16
format, and the witness the batch is built around verifies."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem
from tilefoundry_b200 import problem_to_json
from tilefoundry_b200.batch import FrameSet, PeriodicBatch
from tilefoundry_b200.workloads import absolute_starts, body_batch


@pytest.mark.parametrize("name", ["gemm", "fa"])
def test_calibrated_bodies_cover_the_capacity_check(name):
    problem, packed, witness, frames, batch, kind = body_batch(name, 2000, seed=4, calibrated=True)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    # the witness the neighbourhood is drawn around verifies
    wf = FrameSet(packed)
    f0 = wf.add(witness.lanes, witness.sync)
    one = PeriodicBatch.from_starts(witness.prologue[None, :], witness.offset[None, :], np.array([witness.ii]),
                                    np.array([f0]))
    wp, wo = absolute_starts(one)
    assert oracle.classify_periodic(wp, wo, one.ii, wf.frames, one.frame)[0][0] in (0, 20)
    # the batch: int16 deltas around int32 bases, every class the configs need
    assert batch.prologue_delta.dtype == np.int16 and batch.offset_delta.dtype == np.int16
    p, o = absolute_starts(batch)
    verdict, makespan, _ii = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    classes = set(np.unique(verdict).tolist())
    assert {0, 12, 20} <= classes, classes
    assert 0.1 < float(np.mean(verdict == 0)) < 0.9
    assert (makespan[verdict == 0] > 0).all()
    assert set(np.unique(kind).tolist()) <= {0, 1, 2, 3, 4}
