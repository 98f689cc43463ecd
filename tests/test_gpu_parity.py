"""GPU parity: every candidate's (verdict, makespan, II) from libtfv.so equals the oracle's.

Three sources of truth, in decreasing strength:
* the reference's own verdicts committed under tests/golden/ (make_golden.py),
* the C oracle (pinned to those verdicts by test_oracle.py) on seeded batches of
  every shape the kernels special-case (1, 2, >= 3 iterations; up to 8 lanes; over
  64 operations; resources; loop-carried shared values),
* size-independent properties on full-size batches.
"""

from __future__ import annotations

import numpy as np
import pytest

from golden_data import PROBLEMS, periodic_cases, problem_text, raw_cases
from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem
from random_cases import random_problem, raw_mutations
from tilefoundry_b200 import (
    WarpgroupVerificationError,
    WarpgroupVerifier,
    _verify_warpgroup_schedule,
    pack_problem,
    problem_from_json,
    problem_to_json,
    verify_warpgroup_schedule,
)
from tilefoundry_b200.batch import PeriodicBatch
from tilefoundry_b200.workloads import (
    absolute_starts,
    mla_perturbations,
    neighbourhood,
    shared_producers,
    witness_from_rows,
)

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


@pytest.fixture(scope="module")
def verifiers():
    _torch()
    cache = {}
    yield cache
    for v in cache.values():
        v.close()


def verifier_for(cache, name):
    if name not in cache:
        cache[name] = WarpgroupVerifier(problem_from_json(problem_text(name)))
    return cache[name]


@pytest.mark.parametrize("name", PROBLEMS)
def test_rows_kernel_matches_reference_verdicts(verifiers, name):
    verifier = verifier_for(verifiers, name)
    cases, verdicts = raw_cases(name)
    verdict, makespan, ii = verifier.verify_schedules(cases)
    expected = np.array(verdicts, dtype=np.int64)
    assert np.array_equal(verdict, expected[:, 0])
    assert np.array_equal(makespan, expected[:, 1])
    assert np.array_equal(ii, expected[:, 2])


def _periodic_from_golden(verifier, data):
    frames = verifier.new_frames()
    ids = [frames.add(lanes, sync) for lanes, sync in data["frames"]]
    batch = PeriodicBatch.from_starts(data["prologue"], data["offset"], data["ii"], np.array(ids)[data["frame"]])
    return frames, batch


@pytest.mark.parametrize("name", PROBLEMS)
def test_periodic_host_entry_matches_reference_verdicts(verifiers, name):
    verifier = verifier_for(verifiers, name)
    data = periodic_cases(name)
    frames, batch = _periodic_from_golden(verifier, data)
    verdict, makespan, ii = verifier.verify_periodic(frames, batch)
    assert np.array_equal(verdict, data["verdict"])
    assert np.array_equal(makespan, data["makespan"])
    assert np.array_equal(ii, data["iiv"])


@pytest.mark.parametrize("name", ["mla", "tiny", "resource_c1_w2", "shared_init_i4"])
def test_periodic_device_entry_matches_reference_verdicts(verifiers, name):
    torch = _torch()
    verifier = verifier_for(verifiers, name)
    data = periodic_cases(name)
    frames, batch = _periodic_from_golden(verifier, data)
    dev = torch.device("cuda", verifier.device)
    dframes = verifier.frames_to_device(frames)
    table = verifier.analyze(dframes)
    tensors = {
        key: torch.from_numpy(getattr(batch, key)).to(dev)
        for key in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")
    }
    verdict, makespan, ii = (t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors))
    assert np.array_equal(verdict, data["verdict"])
    assert np.array_equal(makespan, data["makespan"])
    assert np.array_equal(ii, data["iiv"])


def test_mla_perturbation_batch_matches_oracle(verifiers):
    problem = problem_from_json(problem_text("mla"))
    verifier = verifier_for(verifiers, "mla")
    witness = witness_from_rows(verifier.packed, *raw_cases("mla")[0][0])
    frames, batch, _kind = mla_perturbations(verifier.packed, witness, 1 << 16, seed=5, producers=shared_producers(problem))
    verdict, makespan, ii = verifier.verify_periodic(frames, batch)
    oracle = OracleProblem(load_problem(problem_text("mla")))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)


@pytest.mark.parametrize("seed", range(24))
def test_random_problems_periodic_match_oracle(seed):
    problem, packed, witness = random_problem(seed)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    with WarpgroupVerifier(packed) as verifier:
        frames, batch = neighbourhood(packed, witness, 3000, seed=seed, jitter=8)
        verdict, makespan, ii = verifier.verify_periodic(frames, batch)
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)


@pytest.mark.parametrize("seed", range(24))
def test_random_problems_rows_match_oracle(seed):
    problem, packed, witness = random_problem(seed)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    cases = raw_mutations(packed, witness, 300, seed)
    with WarpgroupVerifier(packed) as verifier:
        verdict, makespan, ii = verifier.verify_schedules(cases)
    ov, om, oi = oracle.classify_raw(cases)
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)


def test_domain_limits_and_packing_contract(verifiers):
    verifier = verifier_for(verifiers, "tiny")
    data = periodic_cases("tiny")
    frames, batch = _periodic_from_golden(verifier, data)
    huge = PeriodicBatch(batch.base_prologue, batch.base_offset, batch.prologue_delta[:, :2].copy(),
                         batch.offset_delta[:, :2].copy(), np.array([1 << 29, 3], dtype=np.int32),
                         np.array([0, len(frames) + 5], dtype=np.int32))
    verdict, _, _ = verifier.verify_periodic(frames, huge)
    assert verdict[0] == -1  # (I - 1) * II reaches 2^30: no verdict in the int32 domain
    assert verdict[1] == -2  # frame index outside the frame table
    empty = PeriodicBatch(batch.base_prologue, batch.base_offset, batch.prologue_delta[:, :0].copy(),
                          batch.offset_delta[:, :0].copy(), np.zeros(0, np.int32), np.zeros(0, np.int32))
    assert verifier.verify_periodic(frames, empty)[0].shape == (0,)


def test_drop_in_raises_the_reference_errors():
    """Mirrors test_verifier_requires_fixed_ownership_and_cross_lane_completion_sync (reference tests :272-288)."""
    problem = problem_from_json(problem_text("tiny"))
    packed = pack_problem(problem)
    cases, verdicts = raw_cases("tiny")
    lanes, sync, rows = next(c for c, v in zip(cases, verdicts) if v[0] == 0)
    from tilefoundry_b200 import SCHEDULE_FORMAT, SynchronizationEdge, TimedOperation, WarpgroupLane, WarpgroupSchedule

    def record(lanes, sync, rows):
        return WarpgroupSchedule(SCHEDULE_FORMAT, tuple(WarpgroupLane(tuple(l)) for l in lanes),
                                 tuple(SynchronizationEdge(*e) for e in sync), tuple(TimedOperation(*r) for r in rows))

    _verify_warpgroup_schedule(problem, record(lanes, sync, rows))
    required = ("load", "compute", 0)
    assert required in [tuple(e) for e in sync]
    with pytest.raises(WarpgroupVerificationError, match="no lane/sync path"):
        _verify_warpgroup_schedule(problem, record(lanes, [e for e in sync if tuple(e) != required], rows))
    moved = [list(l) for l in lanes]
    moved[0] = []
    moved[1] = ["load"] + [op for op in lanes[1]]
    with pytest.raises(WarpgroupVerificationError, match="expected warp_group"):
        _verify_warpgroup_schedule(problem, record(moved, sync, rows))
    assert packed.n_ops == 4


def test_mla_example_verifies_through_public_entry():
    """Mirrors test_mla_example_is_one_complete_three_document_workflow (reference tests :478-488)."""
    problem = problem_from_json(problem_text("mla"))
    lanes, sync, rows = raw_cases("mla")[0][0]
    verify_warpgroup_schedule("program", "hardware", (lanes, sync, rows), build=lambda program, hardware: problem)


@pytest.mark.parametrize("n", [1000, 1001, 8, 7, 129])
def test_tma_and_plain_load_paths_agree_with_oracle(verifiers, n):
    """Strides that are multiples of 8 take the TMA-fed kernel, others the plain-load kernel."""
    torch = _torch()
    problem = problem_from_json(problem_text("mla"))
    verifier = verifier_for(verifiers, "mla")
    witness = witness_from_rows(verifier.packed, *raw_cases("mla")[0][0])
    frames, batch, _ = mla_perturbations(verifier.packed, witness, n, seed=n, producers=shared_producers(problem))
    dev = torch.device("cuda", verifier.device)
    dframes = verifier.frames_to_device(frames)
    table = verifier.analyze(dframes)
    tensors = {
        key: torch.from_numpy(getattr(batch, key)).to(dev)
        for key in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")
    }
    verdict, makespan, ii = (t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors))
    oracle = OracleProblem(load_problem(problem_text("mla")))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)


@pytest.mark.parametrize("seed", range(16))
def test_resource_capacity_matches_oracle(seed):
    from random_cases import resource_heavy

    problem, packed, frames, batch = resource_heavy(seed, 4000)
    with WarpgroupVerifier(packed) as verifier:
        verdict, makespan, ii = verifier.verify_periodic(frames, batch)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)


@pytest.mark.parametrize("seed", range(4))
def test_resource_capacity_plain_kernel_matches_oracle(seed):
    """An odd candidate count (stride not a multiple of 8) takes the staged plain-load kernel."""
    from random_cases import resource_heavy

    torch = _torch()
    problem, packed, frames, batch = resource_heavy(100 + seed, 3001)
    with WarpgroupVerifier(packed) as verifier:
        dev = torch.device("cuda", verifier.device)
        dframes = verifier.frames_to_device(frames)
        table = verifier.analyze(dframes)
        tensors = {
            key: torch.from_numpy(getattr(batch, key)).to(dev)
            for key in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")
        }
        verdict, makespan, ii = (t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors))
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)


@pytest.mark.parametrize(
    "seed,n_ops,n_resources,iterations",
    [
        (0, 100, 1, 4),  # TMA kernel, 100 windows on one resource (several per lane)
        (1, 60, 2, 13),
        (2, 300, 2, 5),  # global-read kernel, about 150 windows per resource
        (3, 300, 1, 3),  # 300 windows on one resource: one thread per candidate
        (4, 40, 1, 2),
        (5, 40, 1, 1),
    ],
)
def test_resource_capacity_many_windows_match_oracle(seed, n_ops, n_resources, iterations):
    from random_cases import resource_wide

    problem, packed, frames, batch = resource_wide(seed, 2000, n_ops, n_resources, iterations)
    with WarpgroupVerifier(packed) as verifier:
        verdict, makespan, ii = verifier.verify_periodic(frames, batch)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)
    classes = set(np.unique(ov).tolist())
    assert 20 in classes or iterations == 1


# (body, candidates, calibrated capacities, classes the oracle must report). The nominal GEMM and
# FlashAttention capacities cannot be exceeded by a candidate that keeps its lane, sync and
# relation inequalities, so their capacity checks run on the calibrated variants.
BODY_CASES = [
    ("gemm", 4000, True, {0, 12, 15, 18, 20}),
    ("fa", 4000, True, {0, 12, 15, 18, 20}),
    ("gemm", 4000, False, {0, 5, 12, 15, 18}),
    ("fa", 4000, False, {0, 1, 5, 12, 15, 18}),
    ("dag", 1500, False, {0, 1, 5, 12, 15, 20}),
    ("stress", 256, False, {0, 5, 12, 20}),
]


@pytest.mark.parametrize("name,count,calibrated,required", BODY_CASES,
                         ids=[f"{c[0]}{'-calibrated' if c[2] else ''}" for c in BODY_CASES])
def test_kernel_body_configs_match_oracle(name, count, calibrated, required):
    """The GEMM mainloop, FlashAttention, 256-op DAG and 1024-op stress bodies.

    Software-pipelined candidates (half of them corrupted) whose verdicts cover the capacity
    check (class 20) as well as the lane, sync and relation classes.
    """
    from tilefoundry_b200 import workloads

    problem, packed, _witness, frames, batch, _kind = workloads.body_batch(name, count, seed=3, calibrated=calibrated)
    with WarpgroupVerifier(packed) as verifier:
        verdict, makespan, ii = verifier.verify_periodic(frames, batch)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert required <= set(np.unique(ov).tolist())
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)


def _oracle_rows(problem, frames, batch, ii_values):
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    p, o = absolute_starts(batch)
    arrays, memo = oracle.prepare_frames(frames.frames)  # the frames' answers serve every II row
    return [oracle.classify_periodic(p, o, row, frames.frames, batch.frame, frame_arrays=arrays, memo=memo)
            for row in ii_values]


def _assert_sweep(got, want):
    verdict, makespan, ii = got
    for k, (ov, om, oi) in enumerate(want):
        assert np.array_equal(verdict[k], ov), f"II row {k}"
        assert np.array_equal(makespan[k], om), f"II row {k}"
        assert np.array_equal(ii[k], oi), f"II row {k}"


@pytest.mark.parametrize("n", [4096, 3001])
def test_ii_sweep_matches_oracle_mla(verifiers, n):
    """Each candidate at six IIs of its own (TMA kernel for n = 4096, staged kernel for 3001)."""
    problem = problem_from_json(problem_text("mla"))
    verifier = verifier_for(verifiers, "mla")
    witness = witness_from_rows(verifier.packed, *raw_cases("mla")[0][0])
    frames, batch, _ = mla_perturbations(verifier.packed, witness, n, seed=n + 5, producers=shared_producers(problem))
    shifts = np.array([-40, -10, 0, 7, 30, 200])
    ii_values = (batch.ii[None, :].astype(np.int64) + shifts[:, None]).astype(np.int32)
    got = verifier.verify_periodic_sweep(frames, batch, ii_values)
    _assert_sweep(got, _oracle_rows(problem, frames, batch, ii_values))
    # row k equals a plain verification of the batch at those IIs
    single = PeriodicBatch(batch.base_prologue, batch.base_offset, batch.prologue_delta, batch.offset_delta,
                           ii_values[3].copy(), batch.frame)
    verdict, makespan, ii = verifier.verify_periodic(frames, single)
    assert np.array_equal(verdict, got[0][3]) and np.array_equal(makespan, got[1][3])


def test_ii_sweep_matches_oracle_resources():
    from random_cases import resource_wide
    from tilefoundry_b200.workloads import ii_lower_bound, ii_sweep

    problem, packed, frames, batch = resource_wide(7, 600, 80, 2, 6)
    ii_values = np.repeat(ii_sweep(max(ii_lower_bound(packed), int(batch.ii.min()) // 2), 5)[:, None], 600, axis=1)
    with WarpgroupVerifier(packed) as verifier:
        got = verifier.verify_periodic_sweep(frames, batch, ii_values.astype(np.int32))
    want = _oracle_rows(problem, frames, batch, ii_values)
    _assert_sweep(got, want)
    assert {0, 20} <= set(np.unique(np.concatenate([w[0] for w in want])).tolist())


def test_ii_sweep_stress_body_matches_oracle():
    """The 1024-op stress body: 256 candidates, each at the 16 IIs spread over [II_lb, 2 II_lb]."""
    from tilefoundry_b200 import workloads

    problem, packed, _witness, frames, batch, _kind = workloads.body_batch("stress", 256, seed=11)
    ii_values = np.repeat(workloads.ii_sweep(workloads.ii_lower_bound(packed), 16)[:, None], 256, axis=1)
    with WarpgroupVerifier(packed) as verifier:
        got = verifier.verify_periodic_sweep(frames, batch, ii_values.astype(np.int32))
    want = _oracle_rows(problem, frames, batch, ii_values)
    assert {0, 12, 15, 20} <= set(np.unique(np.concatenate([w[0] for w in want])).tolist())
    _assert_sweep(got, want)


@pytest.mark.parametrize("name", ["mla", "resource_c4_w5", "shared_init_i4", "tiny_free"])
def test_verify_documents_matches_record_path(name):
    """Native document decode + rows kernel equals the record path, rejects included."""
    import json

    from tilefoundry_b200 import SCHEDULE_FORMAT, WarpgroupSerializationError, schedule_from_json
    from tilefoundry_b200.decode import CLASS_DECODE_FAILED

    problem = problem_from_json(problem_text(name))
    cases, _verdicts = raw_cases(name)
    docs = [json.dumps({"format": SCHEDULE_FORMAT, "lanes": [list(l) for l in lanes],
                        "sync": [{"after": a, "before": b, "distance": d} for a, b, d in sync],
                        "times": [list(r) for r in rows]}) for lanes, sync, rows in cases[:300]]
    docs += [d.replace("1", "1.0", 1) for d in docs[:5]]
    with WarpgroupVerifier(pack_problem(problem)) as verifier:
        verdict, makespan, ii = verifier.verify_documents(docs)
        records, index = [], []
        for k, d in enumerate(docs):
            try:
                records.append(schedule_from_json(d))
                index.append(k)
            except WarpgroupSerializationError:
                assert verdict[k] == CLASS_DECODE_FAILED
        rv, rm, ri = verifier.verify_schedules(records)
    assert np.array_equal(verdict[index], rv)
    assert np.array_equal(makespan[index], rm)
    assert np.array_equal(ii[index], ri)
    assert len(index) < len(docs)


def test_outlier_candidates_get_verdicts(verifiers):
    """1% of the candidates lie 10^5 cycles or more from the rest, outside the int16 delta range
    of the batch's base: they are verified in batches of their own (verify_periodic_starts)
    and every candidate matches the oracle."""
    problem = problem_from_json(problem_text("mla"))
    verifier = verifier_for(verifiers, "mla")
    witness = witness_from_rows(verifier.packed, *raw_cases("mla")[0][0])
    n = 20000
    frames, batch, _ = mla_perturbations(verifier.packed, witness, n, seed=31, producers=shared_producers(problem))
    p, o = absolute_starts(batch)
    rng = np.random.default_rng(31)
    out = np.flatnonzero(rng.random(n) < 0.01)
    whole = out[: out.size // 2]  # every start later by 1e5-3e5 cycles (verdicts kept, makespans move)
    shift = rng.integers(1, 4, size=whole.size) * 100000
    p[whole] += shift[:, None]
    o[whole] += shift[:, None]
    one = out[out.size // 2:]  # one operation's starts moved by 1e5 cycles
    ops = rng.integers(0, p.shape[1], size=one.size)
    p[one, ops] += 100000
    o[one, ops] += 100000
    verdict, makespan, ii = verifier.verify_periodic_starts(frames, p, o, batch.ii, batch.frame)
    oracle = OracleProblem(load_problem(problem_text("mla")))
    ov, om, oi = oracle.classify_periodic(p, o, batch.ii, frames.frames, batch.frame)
    assert np.array_equal(verdict, ov)
    assert np.array_equal(makespan, om)
    assert np.array_equal(ii, oi)
    assert (verdict[whole] == 0).any()
