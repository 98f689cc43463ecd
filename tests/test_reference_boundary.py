"""The drop-in boundary takes the reference's own records.

The packer reads problems and schedules only through their attributes, so the reference's
``WarpgroupProblem`` (model.py:377) and ``WarpgroupSchedule`` (model.py:481) records pack into
exactly the tables of this package's mirror records, and the GPU drop-in
(``_verify_warpgroup_schedule``, verify.py:203) gives the reference's verdicts on them. These
tests need the reference package under ``baseline/_ref`` and skip without it.
"""

from __future__ import annotations

import numpy as np
import pytest

import reference_records as ref
from golden_data import PROBLEMS, problem_text, raw_cases
from tilefoundry_b200 import pack_problem, problem_from_json
from tilefoundry_b200.batch import FrameSet, pack_rows

pytestmark = pytest.mark.skipif(not ref.available(), reason="the reference package is not installed in baseline/_ref")

FIELDS = ("op_ids", "iterations", "warp_groups", "issue", "latency", "warp_group", "relations", "carried",
          "register_offsets", "register_ops", "resource_ids", "capacity", "window_offsets", "window_resource",
          "window_amount", "window_duration")


@pytest.mark.parametrize("name", PROBLEMS)
def test_reference_problem_records_pack_like_the_mirror(name):
    text = problem_text(name)
    theirs, ours = pack_problem(ref.problem(text)), pack_problem(problem_from_json(text))
    for field in FIELDS:
        a, b = getattr(theirs, field), getattr(ours, field)
        assert np.array_equal(a, b) if isinstance(a, np.ndarray) else a == b, field


@pytest.mark.parametrize("name", PROBLEMS)
def test_reference_schedule_records_pack_like_raw_candidates(name):
    packed = pack_problem(problem_from_json(problem_text(name)))
    cases, verdicts = raw_cases(name)
    records, raw = [], []
    for case, verdict in zip(cases[:400], verdicts[:400]):
        record = ref.schedule(*case)
        assert (record is None) == (verdict[0] == 1)  # the constructors refuse exactly the class-1 cases
        if record is not None:
            records.append(record)
            raw.append(case)
    fa, fb = FrameSet(packed), FrameSet(packed)
    a = pack_rows(packed, fa, records)
    b = pack_rows(packed, fb, raw)
    for key in ("start", "issue_end", "completion", "row_flags", "override", "override_makespan", "override_ii"):
        assert np.array_equal(getattr(a, key), getattr(b, key)), key
    # the same frame content per candidate (a record's sync edges are sorted, so raw candidates
    # that list a set in another order may be deduplicated into more frames)
    xa, xb = fa.arrays(), fb.arrays()

    def content(x, f):
        s = x["sync_set"][f]
        edges = x["sync_edges"][x["sync_offsets"][s]:x["sync_offsets"][s + 1]]
        return x["lane_pos"][f].tolist(), int(x["lane_count"][f]), int(x["flags"][f]), edges.tolist()

    for c in range(len(records)):
        assert content(xa, a.frame[c]) == content(xb, b.frame[c])


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["mla", "tiny", "resource_c4_w5", "shared_init_i4"])
def test_drop_in_verifies_the_reference_records(name):
    """The GPU drop-in on the reference's records returns the reference's verdicts."""
    from tilefoundry_b200 import WarpgroupVerificationError, _verify_warpgroup_schedule, verify_warpgroup_schedules

    _, _, errors = ref.modules()
    problem = ref.problem(problem_text(name))
    cases, verdicts = raw_cases(name)
    pairs = [(ref.schedule(*c), v) for c, v in zip(cases[:300], verdicts[:300])]
    pairs = [(s, v) for s, v in pairs if s is not None]
    got_v, got_m, got_i = verify_warpgroup_schedules(problem, [s for s, _ in pairs])
    assert np.array_equal(got_v, [v[0] for _, v in pairs])
    assert np.array_equal(got_m, [v[1] for _, v in pairs])
    assert np.array_equal(got_i, [v[2] for _, v in pairs])
    for schedule, verdict in pairs[:20]:
        if verdict[0] == 0:
            _verify_warpgroup_schedule(problem, schedule)
        else:
            with pytest.raises(WarpgroupVerificationError):
                _verify_warpgroup_schedule(problem, schedule)
    del errors
