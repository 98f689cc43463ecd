"""The large-body kernel under load: every CTA cycles through its buffer groups many times.

The parity tests on a few hundred candidates give each CTA at most one tile, so no buffer
group is ever reused. Here batches are large enough for many rounds per group (and, for the
1024-operation body, more producer warps than groups), and each result must equal that of
the same candidates verified in chunks small enough to give every CTA one tile at most, with
no candidate reporting a device timeout; a sample is checked against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.fast import OracleProblem
from oracle.problem_doc import load_problem
from tilefoundry_b200 import WarpgroupVerifier, problem_to_json
from tilefoundry_b200.workloads import absolute_starts, body_batch, ii_lower_bound, ii_sweep

pytestmark = pytest.mark.gpu

KEYS = ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")


def _tensors(torch, batch, lo, hi, dev):
    out = {}
    for k in KEYS:
        a = getattr(batch, k)
        if k in ("prologue_delta", "offset_delta"):
            a = a[:, lo:hi]
        elif k in ("ii", "frame"):
            a = a[lo:hi]
        out[k] = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return out


@pytest.mark.parametrize("name,n,n_ii", [("dag", 40000, 1), ("stress", 4096, 4)])
def test_many_rounds_match_single_tile_chunks(name, n, n_ii):
    import torch

    problem, packed, _w, frames, batch, _kind = body_batch(name, n, seed=17)
    dev = torch.device("cuda", 0)
    sweep = np.repeat(ii_sweep(ii_lower_bound(packed), n_ii)[:, None], n, axis=1).astype(np.int32)
    with WarpgroupVerifier(packed) as verifier:
        dframes = verifier.frames_to_device(frames)
        table = verifier.analyze(dframes)

        def run(lo, hi):
            t = _tensors(torch, batch, lo, hi, dev)
            if n_ii == 1:
                out = verifier.verify_periodic_device(dframes, table, t)
                return [x.cpu().numpy()[None, :] for x in out]
            ii = torch.from_numpy(np.ascontiguousarray(sweep[:, lo:hi])).to(dev)
            return [x.cpu().numpy() for x in verifier.verify_periodic_sweep_device(dframes, table, t, ii)]

        whole = run(0, n)
        for _ in range(2):  # repeated launches agree too
            again = run(0, n)
            for a, b in zip(whole, again):
                assert np.array_equal(a, b)
        chunk = 512
        parts = [run(lo, min(n, lo + chunk)) for lo in range(0, n, chunk)]
    for k in range(3):
        assert np.array_equal(whole[k], np.concatenate([part[k] for part in parts], axis=1))
    assert not (whole[0] == -3).any()
    oracle = OracleProblem(load_problem(problem_to_json(problem)))
    p, o = absolute_starts(batch)
    sample = np.arange(0, n, n // 200)
    arrays, memo = oracle.prepare_frames(frames.frames)
    for k in range(n_ii):
        ii_row = batch.ii[sample] if n_ii == 1 else sweep[k, sample]
        ov, om, oi = oracle.classify_periodic(p[sample], o[sample], ii_row, frames.frames, batch.frame[sample],
                                              frame_arrays=arrays, memo=memo)
        assert np.array_equal(whole[0][k, sample], ov)
        assert np.array_equal(whole[1][k, sample], om)
        assert np.array_equal(whole[2][k, sample], oi)
