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


def _both(verifier, frames, batch):
    import torch

    dev = torch.device("cuda", verifier.device)
    dframes = verifier.frames_to_device(frames)
    table = verifier.analyze(dframes)
    tensors = {k: torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev)
               for k in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")}
    counts = np.bincount(batch.frame, minlength=len(frames))
    top = int(np.argmax(counts))
    plan = verifier.plan(frames, top)
    generic = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors)]
    planned = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors, plan=plan,
                                                                         spec_frame=top)]
    return generic, planned, top


@pytest.mark.parametrize("n", [65536, 1000, 8])
def test_plan_matches_frame_table_kernel_and_oracle_mla(n):
    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    witness = witness_from_rows(packed, *raw_cases("mla")[0][0])
    frames, batch, _ = mla_perturbations(packed, witness, n, seed=n + 11, producers=shared_producers(problem))
    with WarpgroupVerifier(packed) as verifier:
        generic, planned, top = _both(verifier, frames, batch)
        assert "tfv_spec_kernel" in verifier.plan(frames, top).source()
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    sample = np.arange(min(n, 4000))
    p, o = absolute_starts(batch)
    ov, om, oi = oracle.classify_periodic(p[sample], o[sample], batch.ii[sample], frames.frames, batch.frame[sample])
    assert np.array_equal(planned[0][sample], ov)
    assert np.array_equal(planned[1][sample], om)
    assert np.array_equal(planned[2][sample], oi)


@pytest.mark.parametrize("seed", range(16))
def test_plan_matches_frame_table_kernel_random(seed):
    problem, packed, witness = random_problem(seed)
    frames, batch = neighbourhood(packed, witness, 4096, seed=seed + 3, jitter=48)
    with WarpgroupVerifier(packed) as verifier:
        generic, planned, _top = _both(verifier, frames, batch)
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)


@pytest.mark.parametrize("name", ["gemm", "fa", "dag"])
def test_plan_matches_frame_table_kernel_bodies(name):
    from tilefoundry_b200 import workloads

    problem = {"gemm": workloads.gemm_mainloop_problem, "fa": workloads.flash_attention_problem,
               "dag": workloads.dag_problem}[name]()
    packed = pack_problem(problem)
    witness = workloads.list_schedule_witness(packed, seed=1)
    frames, batch = neighbourhood(packed, witness, 2048, seed=9, jitter=64)
    with WarpgroupVerifier(packed) as verifier:
        generic, planned, _top = _both(verifier, frames, batch)
    for g, p in zip(generic, planned):
        assert np.array_equal(g, p)
