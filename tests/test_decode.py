"""Native schedule-document decode (host code of libtfv.so) against the Python decoder.

Every document, valid or not, must be accepted or rejected exactly when
``schedule_from_json`` accepts or raises, and an accepted batch must pack into the same
rows and frames as ``schedule_from_json`` + ``pack_rows``. Documents come from the
golden cases of every problem and from seeded text mutations of them.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from golden_data import PROBLEMS, problem_text, raw_cases
from tilefoundry_b200 import SCHEDULE_FORMAT, WarpgroupSerializationError, pack_problem, problem_from_json, schedule_from_json
from tilefoundry_b200.batch import FrameSet, pack_rows
from tilefoundry_b200.decode import NativeFrameSet, decode_schedule_documents


def _document(lanes, sync, rows) -> str:
    return json.dumps({
        "format": SCHEDULE_FORMAT,
        "lanes": [list(lane) for lane in lanes],
        "sync": [{"after": a, "before": b, "distance": d} for a, b, d in sync],
        "times": [list(r) for r in rows],
    })


def _mutations(text: str, rng: np.random.Generator, count: int) -> list[str]:
    out = []
    edits = [
        lambda t: t.replace(":", "::", 1),
        lambda t: t.replace("0", "0.0", 1),
        lambda t: t.replace("1", "true", 1),
        lambda t: t.replace("2", "123456789012345678901234567890", 1),
        lambda t: t.replace('"lanes"', '"lanes": [], "lanes"', 1),
        lambda t: t.replace('"op', '"\\u006fp', 3),
        lambda t: t.replace('"op', '"\\u00e9p', 1),
        lambda t: t.replace("]]", "]] ", 1) + "  ",
        lambda t: t + "x",
        lambda t: t.replace(SCHEDULE_FORMAT, SCHEDULE_FORMAT + "2"),
        lambda t: t.replace('"distance": 1', '"distance": -1', 1),
        lambda t: t.replace('"distance": 0', '"distance": NaN', 1),
        lambda t: t.replace(", ", ",\n\t", 5),
        lambda t: t.replace('"sync": [', '"sync": [{"after": "a", "before": "a", "distance": 0}, ', 1),
        lambda t: t.replace("[[", "[[\"x\", ", 1),
        lambda t: t.replace("1", "9" * 4400, 1),
    ]
    for _ in range(count):
        t = text
        for _ in range(int(rng.integers(1, 3))):
            roll = rng.random()
            if roll < 0.5:
                t = edits[int(rng.integers(len(edits)))](t)
            elif roll < 0.75 and len(t) > 2:
                k = int(rng.integers(len(t)))
                t = t[:k] + t[k + 1:]
            else:
                k = int(rng.integers(len(t)))
                alphabet = "\"{}[],:-0e.\\ "
                t = t[:k] + alphabet[int(rng.integers(len(alphabet)))] + t[k:]
        out.append(t)
    return out


def _python_reference(packed, docs):
    frames = FrameSet(packed)
    status = np.zeros(len(docs), dtype=np.int32)
    records = []
    for c, d in enumerate(docs):
        try:
            records.append(schedule_from_json(d))
        except WarpgroupSerializationError:
            status[c] = 1
    rows = pack_rows(packed, frames, records) if records else None
    return status, frames, rows


@pytest.mark.parametrize("name", PROBLEMS)
def test_native_decode_matches_python(name):
    problem = problem_from_json(problem_text(name))
    packed = pack_problem(problem)
    rng = np.random.default_rng(len(name))
    cases, _verdicts = raw_cases(name)
    base = [_document(*case) for case in cases[:60]]
    docs = base + [m for text in base[:20] for m in _mutations(text, rng, 12)]
    status_py, frames_py, rows_py = _python_reference(packed, docs)
    native = NativeFrameSet(packed)
    decoded = decode_schedule_documents(native, docs, threads=4)
    assert np.array_equal(decoded.status, status_py)
    assert 0 < int(status_py.sum()) < len(docs)
    ok = np.flatnonzero(decoded.status == 0)
    r = decoded.rows
    for key in ("start", "issue_end", "completion", "frame", "row_flags", "override", "override_makespan", "override_ii"):
        assert np.array_equal(getattr(r, key)[ok], getattr(rows_py, key)), key
    assert np.all(r.frame[decoded.status == 1] == -1)
    py, nat = frames_py.arrays(), native.arrays()
    for key in py:
        assert np.array_equal(py[key], nat[key]), key
    native.close()


def test_native_decode_frames_accumulate_across_calls():
    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    docs = [_document(*case) for case in raw_cases("mla")[0][:30]]
    native = NativeFrameSet(packed)
    first = decode_schedule_documents(native, docs[:15])
    second = decode_schedule_documents(native, docs[15:])
    frames_py = FrameSet(packed)
    _status, frames_py, rows_py = _python_reference(packed, docs)
    both = np.concatenate([first.rows.frame, second.rows.frame])
    assert np.array_equal(both[np.concatenate([first.status, second.status]) == 0], rows_py.frame)
    assert len(native) == len(frames_py)


def test_decoders_match_the_reference_decoder():
    """Both decoders accept exactly the documents the reference's warpgroup_schedule_from_json
    accepts (serialization.py:679-727) and decode them to the records it decoded. The fixture
    holds the reference's own outcomes for golden documents and seeded mutations of them
    (tests/golden/make_decode_golden.py ran the reference decoder)."""
    import gzip

    from golden_data import GOLDEN
    from tilefoundry_b200.batch import schedule_parts

    with gzip.open(GOLDEN / "decode_cases.json.gz", "rt", encoding="utf-8") as handle:
        payload = json.load(handle)
    names = sorted(set(payload["problem"]))
    assert names == sorted(PROBLEMS)
    for name in names:
        pick = [k for k, p in enumerate(payload["problem"]) if p == name]
        docs = [payload["document"][k] for k in pick]
        accepted = np.array([payload["outcome"][k] == "accepted" for k in pick])
        decoded = [payload["decoded"][k] for k in pick]
        assert set(payload["outcome"][k] for k in pick) <= {"accepted", "WarpgroupSerializationError"}
        # the Python decoder: same accept/reject, same records
        for doc, ok, want in zip(docs, accepted, decoded):
            try:
                lanes, sync, rows = schedule_parts(schedule_from_json(doc))
            except WarpgroupSerializationError:
                assert not ok
                continue
            assert ok
            assert [list(l) for l in lanes] == want[0]
            assert [list(e) for e in sync] == want[1]
            assert [list(r) for r in rows] == want[2]
        # the native decoder: same accept/reject, and rows and frames equal to packing the
        # reference's decoded records
        packed = pack_problem(problem_from_json(problem_text(name)))
        native = NativeFrameSet(packed)
        got = decode_schedule_documents(native, docs, threads=4)
        assert np.array_equal(got.status == 0, accepted)
        frames = FrameSet(packed)
        ref_rows = pack_rows(packed, frames, [(d[0], [tuple(e) for e in d[1]], [tuple(r) for r in d[2]])
                                              for d, ok in zip(decoded, accepted) if ok])
        ok = np.flatnonzero(accepted)
        for key in ("start", "issue_end", "completion", "frame", "row_flags", "override", "override_makespan",
                    "override_ii"):
            assert np.array_equal(getattr(got.rows, key)[ok], getattr(ref_rows, key)), (name, key)
        ours, theirs = native.arrays(), frames.arrays()
        for key in ours:
            assert np.array_equal(ours[key], theirs[key]), (name, key)
        native.close()
