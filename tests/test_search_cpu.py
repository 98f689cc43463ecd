"""Host side of the neighbourhood search (search.py), on the CPU: the neighbours drawn by
`_device_neighbours` (torch on any device) form a valid periodic batch around the incumbent,
the lane-move frames keep the incumbent first, and the objective orders (II, makespan)
lexicographically. The oracle checks that the neighbourhood holds verified schedules."""

from __future__ import annotations

import numpy as np
import torch

from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem
from tilefoundry_b200 import pack_problem, problem_to_json
from tilefoundry_b200.search import _device_neighbours, _lane_moves, _objective
from tilefoundry_b200.workloads import list_schedule_witness, random_dag_problem


def _setup():
    problem = random_dag_problem(24, layers=4, lanes=3, n_resources=2, iterations=6, seed=3, latency=(4, 80),
                                 capacity=(6, 20))
    packed = pack_problem(problem)
    return problem, packed, list_schedule_witness(packed, seed=1)


def _draw(witness, n, n_frames, seed, step):
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    return _device_neighbours(torch, witness, n, n_frames, gen, step, torch.device("cpu"))


def test_neighbours_form_a_valid_periodic_batch():
    _problem, packed, witness = _setup()
    n, n_frames, step = 4096, 9, max(1, witness.ii // 16)
    cand = _draw(witness, n, n_frames, 11, step)
    N = packed.n_ops
    assert cand["prologue_delta"].shape == (N, n) and cand["prologue_delta"].dtype == torch.int16
    assert cand["offset_delta"].shape == (N, n) and cand["offset_delta"].dtype == torch.int16
    assert cand["ii"].dtype == torch.int32 and cand["frame"].dtype == torch.int32
    ii = cand["ii"].numpy().astype(np.int64)
    assert ii.min() >= 1 and ii.max() <= witness.ii
    frame = cand["frame"].numpy()
    assert frame.min() >= 0 and frame.max() < n_frames
    p = cand["base_prologue"].numpy()[:, None].astype(np.int64) + cand["prologue_delta"].numpy()
    o = cand["base_offset"].numpy()[:, None].astype(np.int64) + cand["offset_delta"].numpy()
    assert (p >= 0).all() and (o + ii[None, :] >= 0).all()  # iteration 0 and the first body start
    assert (p <= witness.prologue[:, None]).all() and (o <= witness.offset[:, None]).all()  # pulled earlier only
    again = _draw(witness, n, n_frames, 11, step)
    assert all(torch.equal(cand[k], again[k]) for k in cand)  # seeded
    other = _draw(witness, n, n_frames, 12, step)
    assert not torch.equal(cand["prologue_delta"], other["prologue_delta"])


def test_lane_moves_keep_the_incumbent_first():
    _problem, packed, witness = _setup()
    frames = _lane_moves(packed, witness, np.random.default_rng(5), count=16)
    assert frames.frames[0] == frames.frames[frames.add(witness.lanes, witness.sync)]
    assert 2 <= len(frames) <= 17
    for lanes, _sync in frames.frames:  # every frame places every operation exactly once
        placed = sorted(op for lane in lanes for op in lane)
        assert placed == sorted(packed.op_ids)


def test_objective_is_lexicographic():
    ii = np.array([5, 5, 4, 4])
    makespan = np.array([100, 90, 1000, 999])
    keys = _objective(ii, makespan, iterations=6)
    assert list(np.argsort(keys)) == [3, 2, 1, 0]
    flat = _objective(ii, makespan, iterations=2)  # no II below three iterations: makespan alone
    assert list(np.argsort(flat)) == [1, 0, 3, 2]


def test_the_neighbourhood_holds_verified_schedules():
    problem, packed, witness = _setup()
    frames = _lane_moves(packed, witness, np.random.default_rng(5), count=8)
    cand = _draw(witness, 2048, len(frames), 7, max(1, witness.ii // 16))
    p = (cand["base_prologue"].numpy()[None, :].astype(np.int64) + cand["prologue_delta"].numpy().T)
    o = (cand["base_offset"].numpy()[None, :].astype(np.int64) + cand["offset_delta"].numpy().T)
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    verdict, _makespan, _ii = oracle.classify_periodic(p, o, cand["ii"].numpy(), frames.frames, cand["frame"].numpy())
    assert (verdict == 0).any()  # the search has somewhere to go
    assert (verdict != 0).any()  # and the oracle rejects some of the draws
