"""Failure detection on the GPU without a fault: bounded device waits that run out.

The ring kernel (generated plans) and the large-body kernel hand tiles between warps through
mbarriers and tags; every such wait is bounded in time (tfv_set_device_wait_limit, one second
by default). With the limit at zero a waiting warp gives up at its first unsuccessful test:
its CTA stops, the candidates it has not verified report TFV_CLASS_DEVICE_TIMEOUT (-3), and the
launch ends normally. The candidates that were verified before the CTA stopped keep their exact
results, and the next launch with the default limit on the same device is exact again.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from golden_data import problem_text, raw_cases
from tilefoundry_b200 import WarpgroupVerifier, _lib, pack_problem, problem_from_json
from tilefoundry_b200.workloads import body_batch, mla_perturbations, shared_producers, witness_from_rows

pytestmark = pytest.mark.gpu

TIMEOUT = -3


def _set_limit(ns: int) -> int:
    previous = ctypes.c_uint64()
    assert _lib.load().tfv_set_device_wait_limit(ns, ctypes.byref(previous)) == 0
    return int(previous.value)


def _device(verifier, frames, batch):
    import torch

    dev = torch.device("cuda", verifier.device)
    dframes = verifier.frames_to_device(frames)
    tensors = {k: torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev)
               for k in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")}
    return dframes, tensors


def _check_timeouts(expected, timed_out_run, again):
    verdict = timed_out_run[0]
    hit = verdict == TIMEOUT
    assert hit.any(), "a zero wait limit must make some waits give up"
    for got, want in zip(timed_out_run, expected):  # verified candidates keep exact results
        assert np.array_equal(got[~hit], want[~hit])
    assert np.array_equal(timed_out_run[1][hit], np.zeros(int(hit.sum())))
    for got, want in zip(again, expected):  # the device is usable and exact afterwards
        assert np.array_equal(got, want)


def test_large_body_kernel_waits_give_up_and_recover():
    import torch

    problem, packed, _w, frames, batch, _kind = body_batch("dag", 30000, seed=5)
    with WarpgroupVerifier(packed) as verifier:
        dframes, tensors = _device(verifier, frames, batch)
        table = verifier.analyze(dframes)
        expected = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors)]
        assert TIMEOUT not in expected[0]
        previous = _set_limit(0)
        try:
            timed_out = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors)]
        finally:
            _set_limit(previous)
        torch.cuda.synchronize()
        again = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors)]
    _check_timeouts(expected, timed_out, again)


def test_ring_plan_waits_give_up_and_recover():
    import torch

    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    witness = witness_from_rows(packed, *raw_cases("mla")[0][0])
    frames, batch, _ = mla_perturbations(packed, witness, 1 << 20, seed=21, producers=shared_producers(problem))
    with WarpgroupVerifier(packed) as verifier:
        dframes, tensors = _device(verifier, frames, batch)
        table = verifier.analyze(dframes)
        top = int(np.argmax(np.bincount(batch.frame, minlength=len(frames))))
        plan = verifier.plan(frames, top, kernel="ring")
        expected = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors, plan=plan,
                                                                             spec_frame=top)]
        assert TIMEOUT not in expected[0]
        previous = _set_limit(0)
        try:
            timed_out = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors, plan=plan,
                                                                                  spec_frame=top)]
        finally:
            _set_limit(previous)
        torch.cuda.synchronize()
        again = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors, plan=plan,
                                                                           spec_frame=top)]
    _check_timeouts(expected, timed_out, again)
