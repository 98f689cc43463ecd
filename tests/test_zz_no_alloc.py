"""The allocation-free entry point returns exactly what the allocating path returns.

Callers that own no device memory of their own — a search process living inside a host
framework whose pooled allocator holds the GPU, or a latency-sensitive caller that must
not call cudaMalloc/cudaFree because those can synchronize the device — use
``tfv_verify_periodic_static``, whose frame table is a static device array instead of a
buffer the caller allocates. This test calls it twice in a row through the C ABI, on two
different batches, and compares each result with ``tfv_analyze_frames`` +
``tfv_verify_periodic`` on a caller-allocated table. It also checks that frames needing
more than the static table's capacity are refused.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from golden_data import problem_text, raw_cases
from tilefoundry_b200 import WarpgroupVerifier, _lib, problem_from_json
from tilefoundry_b200.workloads import mla_perturbations, shared_producers, witness_from_rows

pytestmark = pytest.mark.gpu

BATCH_KEYS = ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")


def _device_batch(torch, batch, dev):
    tensors = {key: torch.from_numpy(np.ascontiguousarray(getattr(batch, key))).to(dev) for key in BATCH_KEYS}
    struct = _lib.PeriodicBatch(
        int(tensors["ii"].shape[0]), int(tensors["prologue_delta"].stride(0)),
        *(tensors[key].data_ptr() for key in BATCH_KEYS),
    )
    return tensors, struct


def test_static_entry_matches_allocating_entry_on_two_calls():
    import torch

    assert torch.cuda.is_available()
    problem = problem_from_json(problem_text("mla"))
    with WarpgroupVerifier(problem, device=0) as verifier:
        dev = torch.device("cuda", 0)
        lib = _lib.load()
        witness = witness_from_rows(verifier.packed, *raw_cases("mla")[0][0])
        for seed, n in ((101, 50_000), (202, 4099)):
            frames, batch, _ = mla_perturbations(verifier.packed, witness, n, seed=seed, producers=shared_producers(problem))
            dframes = verifier.frames_to_device(frames)
            tensors, bstruct = _device_batch(torch, batch, dev)
            table = verifier.analyze(dframes)
            expected = [t.cpu().numpy() for t in verifier.verify_periodic_device(dframes, table, tensors)]
            out = tuple(torch.full((n,), -7, dtype=torch.int32, device=dev) for _ in range(3))
            results = _lib.Results(*(t.data_ptr() for t in out))
            stream = torch.cuda.current_stream(dev).cuda_stream
            status = lib.tfv_verify_periodic_static(
                verifier._handle, ctypes.byref(dframes.struct), ctypes.byref(bstruct), ctypes.byref(results), stream
            )
            assert status == 0, _lib.last_error()
            torch.cuda.synchronize(dev)
            for got, want in zip(out, expected):
                assert np.array_equal(got.cpu().numpy(), want)

        # Frames whose table would exceed the static array are refused before any launch.
        oversized = _lib.Frames.from_buffer_copy(dframes.struct)
        oversized.n_frames = 1 << 20
        status = lib.tfv_verify_periodic_static(
            verifier._handle, ctypes.byref(oversized), ctypes.byref(bstruct), ctypes.byref(results), stream
        )
        assert status == -4
        assert "static table" in _lib.last_error()
