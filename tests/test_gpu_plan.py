"""Frame-specialised kernels (tfv_plan_*, generated and compiled at run time) give the
same verdicts, makespans and IIs as the frame-table kernel, and as the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from golden_data import problem_text, raw_cases
from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem
from random_cases import random_problem
from tilefoundry_b200 import WarpgroupVerifier, pack_problem, problem_from_json, problem_to_json
from tilefoundry_b200.workloads import (
    absolute_starts,
    mla_perturbations,
    neighbourhood,
    shared_producers,
    witness_from_rows,
)

pytestmark = pytest.mark.gpu


def _both(verifier, frames, batch, kernel="auto", ring_warps=0, misalign=False):
    """Frame-table kernel and plan on the same batch. misalign: the frame and II arrays
    start 4 bytes past a 16-byte boundary (the ring then stages them with plain loads)."""
    import torch

    dev = torch.device("cuda", verifier.device)
    dframes = verifier.frames_to_device(frames)
    table = verifier.analyze(dframes)
    tensors = {k: torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev)
               for k in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")}
    if misalign:
        for k in ("ii", "frame"):
            shifted = torch.empty(tensors[k].numel() + 1, dtype=tensors[k].dtype, device=dev)[1:]
            shifted.copy_(tensors[k])
            assert shifted.data_ptr() % 16 == 4
            tensors[k] = shifted
    counts = np.bincount(batch.frame, minlength=len(frames))
    top = int(np.argmax(counts))
    plan = verifier.plan(frames, top, kernel=kernel, ring_warps=ring_warps)
    if kernel != "auto":
        assert plan.kernel == kernel
    generic = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors)]
    planned = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors, plan=plan,
                                                                         spec_frame=top)]
    return generic, planned, top


@pytest.mark.parametrize("kernel", ["ring", "tiles"])
@pytest.mark.parametrize("n", [65536, 1000, 8])
def test_plan_matches_frame_table_kernel_and_oracle_mla(n, kernel):
    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    witness = witness_from_rows(packed, *raw_cases("mla")[0][0])
    frames, batch, _ = mla_perturbations(packed, witness, n, seed=n + 11, producers=shared_producers(problem))
    with WarpgroupVerifier(packed) as verifier:
        generic, planned, top = _both(verifier, frames, batch, kernel=kernel)
        name = "tfv_spec_ring" if kernel == "ring" else "tfv_spec_kernel"
        assert name in verifier.plan(frames, top, kernel=kernel).source()
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    sample = np.arange(min(n, 4000))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p[sample], o[sample], batch.ii[sample], frames.frames, batch.frame[sample])
    assert np.array_equal(planned[0][sample], ov)
    assert np.array_equal(planned[1][sample], om)
    assert np.array_equal(planned[2][sample], oi)


@pytest.mark.parametrize("seed,kernel", [(seed, "auto") for seed in range(10)] + [(seed, "tiles") for seed in range(6)])
def test_plan_matches_frame_table_kernel_random(seed, kernel):
    problem, packed, witness = random_problem(seed)
    frames, batch = neighbourhood(packed, witness, 4096, seed=seed + 3, jitter=48)
    with WarpgroupVerifier(packed) as verifier:
        generic, planned, _top = _both(verifier, frames, batch, kernel=kernel)
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)


@pytest.mark.parametrize("ring_warps,misalign", [(1, False), (7, True), (31, True), (16, False)])
def test_ring_plan_warps_and_unaligned_frames(ring_warps, misalign):
    """Any consumer-warp count, and frame/II arrays off a 16-byte boundary, give the same results."""
    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    witness = witness_from_rows(packed, *raw_cases("mla")[0][0])
    frames, batch, _ = mla_perturbations(packed, witness, 20000 + 8 * ring_warps, seed=ring_warps,
                                         producers=shared_producers(problem))
    with WarpgroupVerifier(packed) as verifier:
        generic, planned, _top = _both(verifier, frames, batch, kernel="ring", ring_warps=ring_warps,
                                       misalign=misalign)
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)


def test_ring_plan_unsupported_when_slots_do_not_fit():
    """A 256-operation body leaves no room for three ring slots: the ring is refused before
    any compilation (the automatic choice then takes the tiles kernel, see the DAG body)."""
    from tilefoundry_b200 import workloads
    from tilefoundry_b200.errors import VerifierRuntimeError

    packed = pack_problem(workloads.dag_problem())
    witness = workloads.list_schedule_witness(packed, seed=1)
    frames, _batch = neighbourhood(packed, witness, 16, seed=2, jitter=8)
    with WarpgroupVerifier(packed) as verifier:
        with pytest.raises(VerifierRuntimeError):
            verifier.plan(frames, 0, kernel="ring")


@pytest.mark.parametrize("name", ["gemm", "fa", "dag"])
def test_plan_matches_frame_table_kernel_bodies(name):
    from tilefoundry_b200 import workloads

    problem = {"gemm": workloads.gemm_mainloop_problem, "fa": workloads.flash_attention_problem,
               "dag": workloads.dag_problem}[name]()
    packed = pack_problem(problem)
    witness = workloads.list_schedule_witness(packed, seed=1)
    frames, batch = neighbourhood(packed, witness, 2048, seed=9, jitter=64)
    with WarpgroupVerifier(packed) as verifier:
        generic, planned, top = _both(verifier, frames, batch)
        plan = verifier.plan(frames, top)  # the plan _both built (cached per frame content)
        # DAG: 256 operations leave no room for three ring slots and exceed the delta masks
        assert (plan.kernel, plan.delta) == (("tiles", False) if name == "dag" else ("ring", True))
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)


def test_plan_with_another_frames_index_takes_the_frame_table_path():
    """A spec_frame that names a frame other than the plan's is detected on the device: every
    candidate then takes the frame-table path and the results stay exact. An index outside
    the frames is refused."""
    import torch

    from tilefoundry_b200.errors import VerifierRuntimeError

    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    witness = witness_from_rows(packed, *raw_cases("mla")[0][0])
    frames, batch, _ = mla_perturbations(packed, witness, 20000, seed=77, producers=shared_producers(problem))
    with WarpgroupVerifier(packed) as verifier:
        dev = torch.device("cuda", verifier.device)
        dframes = verifier.frames_to_device(frames)
        table = verifier.analyze(dframes)
        tensors = {k: torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev)
                   for k in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")}
        counts = np.bincount(batch.frame, minlength=len(frames))
        top = int(np.argmax(counts))
        other = int(np.argsort(counts)[-2])
        assert frames.frames[other] != frames.frames[top]
        generic = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors)]
        for delta in (True, False):
            plan = verifier.plan(frames, top, delta=delta)
            wrong = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors, plan=plan,
                                                                               spec_frame=other)]
            for g, w in zip(generic, wrong):
                assert np.array_equal(g, w)
            with pytest.raises(VerifierRuntimeError):
                verifier.verify_periodic_device(dframes, table, tensors, plan=plan, spec_frame=len(frames))


def test_ring_plan_warp_count_and_kernel_timing():
    """The default ring plan keeps its values in registers at one of the warp counts the
    library tries, and with timing on records one event pair per call around the generated
    kernel (positive, shorter than the whole call)."""
    import torch

    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    witness = witness_from_rows(packed, *raw_cases("mla")[0][0])
    frames, batch, _ = mla_perturbations(packed, witness, 1 << 20, seed=5, producers=shared_producers(problem))
    with WarpgroupVerifier(packed) as verifier:
        dev = torch.device("cuda", verifier.device)
        dframes = verifier.frames_to_device(frames)
        table = verifier.analyze(dframes)
        tensors = {k: torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev)
                   for k in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")}
        top = int(np.argmax(np.bincount(batch.frame, minlength=len(frames))))
        plan = verifier.plan(frames, top)
        assert plan.kernel == "ring" and plan.ring_warps in (19, 15, 11)
        assert verifier.plan(frames, top, ring_warps=7).ring_warps == 7
        assert plan.kernel_times() == []
        plan.set_timing(True)
        begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record()
        results = [verifier.verify_periodic_device(dframes, table, tensors, plan=plan, spec_frame=top)
                   for _ in range(3)]
        end.record()
        torch.cuda.synchronize(dev)
        plan.set_timing(False)
        times = plan.kernel_times()
        assert len(times) == 3 and all(0 < t for t in times)
        assert sum(times) < begin.elapsed_time(end)
        assert plan.kernel_times() == []  # read once
        verifier.verify_periodic_device(dframes, table, tensors, plan=plan, spec_frame=top)
        torch.cuda.synchronize(dev)
        assert plan.kernel_times() == []  # timing off: nothing recorded
        for r in results[1:]:
            assert all(torch.equal(a, b) for a, b in zip(results[0], r))
