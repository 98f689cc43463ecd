"""Delta verification of frame-specialised plans (tfv_plan_delta).

With delta verification the generated code records which of the plan frame's lane and
sync edges a candidate violates; every frame that shares all but a few edges with the plan
frame runs that code too (its kept edges as a mask, its added edges as program entries),
and frames that differ more take the frame-table path. Every case compares the plan with
the frame-table kernel on the same batch, and a sample with the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from golden_data import problem_text, raw_cases
from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem
from random_cases import random_problem
from tilefoundry_b200 import WarpgroupVerifier, pack_problem, problem_from_json, problem_to_json
from tilefoundry_b200.batch import FrameSet, PeriodicBatch
from tilefoundry_b200.workloads import (
    absolute_starts,
    mla_perturbations,
    neighbourhood,
    shared_producers,
    witness_from_rows,
)

pytestmark = pytest.mark.gpu


def _mla():
    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    witness = witness_from_rows(packed, *raw_cases("mla")[0][0])
    return problem, packed, witness


def _device_batch(verifier, batch):
    import torch

    dev = torch.device("cuda", verifier.device)
    return {k: torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev)
            for k in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")}


def _generic_and_planned(verifier, frames, batch, plan, spec_frame):
    dframes = verifier.frames_to_device(frames)
    table = verifier.analyze(dframes)
    tensors = _device_batch(verifier, batch)
    generic = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors)]
    planned = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors, plan=plan,
                                                                         spec_frame=spec_frame)]
    return generic, planned


def _check_oracle(problem, frames, batch, planned, count=3000):
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    sample = np.arange(min(batch.n, count))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p[sample], o[sample], batch.ii[sample], frames.frames, batch.frame[sample])
    assert np.array_equal(planned[0][sample], ov)
    assert np.array_equal(planned[1][sample], om)
    assert np.array_equal(planned[2][sample], oi)


@pytest.mark.parametrize("kernel", ["ring", "tiles"])
def test_delta_mixes_edge_frames_and_generic_frames(kernel):
    """Frames with every lane reversed (every successor changes) or a disjoint sync program
    exceed the added-edge budget and take the frame-table path, in the same tiles as frames
    described by edges."""
    problem, packed, witness = _mla()
    n = 16384
    frames, batch, _ = mla_perturbations(packed, witness, n, seed=5, producers=shared_producers(problem))
    reversed_lanes = frames.add([list(reversed(lane)) for lane in witness.lanes], witness.sync)
    shifted_sync = frames.add(witness.lanes, [(a, b, d + 1) for (a, b, d) in witness.sync])
    rng = np.random.default_rng(3)
    frame = batch.frame.copy()
    pick = np.flatnonzero(rng.random(n) < 0.1)
    frame[pick] = rng.choice(np.array([reversed_lanes, shifted_sync], dtype=np.int32), size=pick.size)
    batch = PeriodicBatch(batch.base_prologue, batch.base_offset, batch.prologue_delta, batch.offset_delta,
                          batch.ii, frame)
    top = int(np.argmax(np.bincount(batch.frame, minlength=len(frames))))
    with WarpgroupVerifier(packed) as verifier:
        plan = verifier.plan(frames, top, kernel=kernel)
        assert plan.delta and plan.kernel == kernel
        generic, planned = _generic_and_planned(verifier, frames, batch, plan, top)
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)
    _check_oracle(problem, frames, batch, planned)


def test_delta_plan_reused_across_frame_sets():
    """One plan serves frame sets of different sizes that hold its frame at different
    indices (its device table grows with the frame count)."""
    problem, packed, witness = _mla()
    small = FrameSet(packed)
    small.add(witness.lanes, witness.sync)
    with WarpgroupVerifier(packed) as verifier:
        plan = verifier.plan(small, 0)
        assert plan.delta
        for n, seed in ((256, 1), (8192, 2)):
            frames, batch, _ = mla_perturbations(packed, witness, n, seed=seed, producers=shared_producers(problem))
            if n == 256:  # the one-frame set first, then one of 132 frames
                frames = small
                batch = PeriodicBatch(batch.base_prologue, batch.base_offset, batch.prologue_delta,
                                      batch.offset_delta, batch.ii, np.zeros(n, dtype=np.int32))
            spec = frames.add(witness.lanes, witness.sync)
            generic, planned = _generic_and_planned(verifier, frames, batch, plan, spec)
            for g, p in zip(generic, planned):
                assert np.array_equal(g, p)


@pytest.mark.parametrize("kernel", ["ring", "tiles"])
def test_min_form_plans(kernel):
    """Plans built without delta verification (the plan frame's candidates only)."""
    problem, packed, witness = _mla()
    frames, batch, _ = mla_perturbations(packed, witness, 8192, seed=9, producers=shared_producers(problem))
    top = int(np.argmax(np.bincount(batch.frame, minlength=len(frames))))
    with WarpgroupVerifier(packed) as verifier:
        plan = verifier.plan(frames, top, kernel=kernel, delta=False)
        assert not plan.delta and plan.kernel == kernel
        generic, planned = _generic_and_planned(verifier, frames, batch, plan, top)
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)
    _check_oracle(problem, frames, batch, planned, count=1500)


@pytest.mark.parametrize("seed", range(4))
def test_delta_random_problems_plan_of_a_minor_frame(seed):
    """The plan's frame need not be the most frequent one: a minor variant as the plan
    frame makes the base frame itself a delta frame (I = 1, 2 and >= 3 all occur)."""
    problem, packed, witness = random_problem(seed + 40)
    frames, batch = neighbourhood(packed, witness, 4096, seed=seed, jitter=40)
    counts = np.bincount(batch.frame, minlength=len(frames))
    minor = int(np.argsort(counts)[len(counts) // 2])
    with WarpgroupVerifier(packed) as verifier:
        plan = verifier.plan(frames, minor)
        generic, planned = _generic_and_planned(verifier, frames, batch, plan, minor)
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)


def test_back_to_back_calls_with_different_bases():
    """Two planned verifications enqueued on one stream before either result is read, with
    different base starts: the second call's constants (computed on the plan's side stream)
    must not reach the constant bank while the first call's kernel runs."""
    import torch

    problem, packed, witness = _mla()
    frames, batch, _ = mla_perturbations(packed, witness, 65536, seed=21, producers=shared_producers(problem))
    top = int(np.argmax(np.bincount(batch.frame, minlength=len(frames))))
    # the same candidates against bases shifted by 7: every delta moves by -7
    shifted = PeriodicBatch(batch.base_prologue + 7, batch.base_offset + 7,
                            (batch.prologue_delta.astype(np.int32) - 7).astype(np.int16),
                            (batch.offset_delta.astype(np.int32) - 7).astype(np.int16), batch.ii, batch.frame)
    with WarpgroupVerifier(packed) as verifier:
        plan = verifier.plan(frames, top)
        dframes = verifier.frames_to_device(frames)
        table = verifier.analyze(dframes)
        first = _device_batch(verifier, batch)
        second = _device_batch(verifier, shifted)
        dev = torch.device("cuda", verifier.device)
        outs = [tuple(torch.empty(batch.n, dtype=torch.int32, device=dev) for _ in range(3)) for _ in range(2)]
        for _ in range(3):  # both calls in flight together, several times
            verifier.verify_periodic_device(dframes, table, first, out=outs[0], plan=plan, spec_frame=top)
            verifier.verify_periodic_device(dframes, table, second, out=outs[1], plan=plan, spec_frame=top)
        torch.cuda.synchronize(dev)
        generic = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, first)]
    for out in outs:
        for g, p in zip(generic, (t.cpu().numpy() for t in out)):
            assert np.array_equal(g, p)
