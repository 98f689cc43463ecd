"""The oracle is pinned to the reference: every committed reference verdict must be reproduced.

The fixtures under tests/golden/ were produced by running the reference's own
``_verify_warpgroup_schedule`` (tests/golden/make_golden.py). Both restatements
— the step-by-step Python port and the C oracle — must agree with every one.
"""

from __future__ import annotations

import numpy as np
import pytest

from golden_data import PROBLEMS, periodic_cases, problem_text, raw_cases
from oracle import verify_port as port
from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem


@pytest.mark.parametrize("name", PROBLEMS)
def test_c_oracle_matches_reference_raw(name):
    problem = load_problem(problem_text(name))
    cases, verdicts = raw_cases(name)
    verdict, makespan, ii = OracleProblem(problem).classify_raw(cases)
    expected = np.array(verdicts, dtype=np.int64)
    assert np.array_equal(verdict, expected[:, 0])
    assert np.array_equal(makespan, expected[:, 1])
    assert np.array_equal(ii, expected[:, 2])


@pytest.mark.parametrize("name", PROBLEMS)
def test_c_oracle_matches_reference_periodic(name):
    problem = load_problem(problem_text(name))
    data = periodic_cases(name)
    verdict, makespan, ii = OracleProblem(problem).classify_periodic(
        data["prologue"], data["offset"], data["ii"], data["frames"], data["frame"]
    )
    assert np.array_equal(verdict, data["verdict"])
    assert np.array_equal(makespan, data["makespan"])
    assert np.array_equal(ii, data["iiv"])


@pytest.mark.parametrize("name", [p for p in PROBLEMS if p != "mla"])
def test_python_port_matches_reference_raw(name):
    problem = load_problem(problem_text(name))
    cases, verdicts = raw_cases(name)
    for case, expected in zip(cases, verdicts):
        assert port.classify(problem, *case) == expected


def test_python_port_matches_reference_on_mla_failures():
    """The MLA cases that fail early (the port takes seconds per passing MLA schedule)."""
    problem = load_problem(problem_text("mla"))
    cases, verdicts = raw_cases("mla")
    checked = 0
    for case, expected in zip(cases, verdicts):
        if expected[0] in (1, 2, 4, 5, 7, 8, 9, 11, 13, 14):
            assert port.classify(problem, *case) == expected
            checked += 1
    assert checked >= 10


def test_python_port_cycle_check_restates_kahn():
    """Class 21 is unreachable after classes 12/15/17/19 pass; the check itself still works."""
    nodes = {(0, "a"), (0, "b")}
    with pytest.raises(port.OracleFailure) as failure:
        port.require_acyclic(nodes, {((0, "a"), (0, "b")), ((0, "b"), (0, "a"))})
    assert failure.value.class_id == port.CYCLE
    port.require_acyclic(nodes, {((0, "a"), (0, "b"))})


def test_golden_covers_every_reachable_class():
    seen = set()
    for name in PROBLEMS:
        seen.update(v[0] for v in raw_cases(name)[1])
        seen.update(int(v) for v in periodic_cases(name)["verdict"])
    assert seen >= {0, 1, 2, 4, 5, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17, 18, 19, 20}


def test_port_export_reproduces_the_reference_exported_mla_sync():
    """The committed MLA schedule was exported by the reference (sync.py:21-62): exporting
    its lanes and times again keeps exactly its 48 sync edges."""
    problem = load_problem(problem_text("mla"))
    lanes, sync, rows = raw_cases("mla")[0][0]
    clanes, csync, crows = port.construct(lanes, sync, rows)
    status, kept = port.export_sync(problem, clanes, crows)
    assert status == "ok"
    assert sorted(kept) == sorted(csync) and len(kept) == 48
