"""Canonical synchronization export on the GPU (drop-in for ``sync.py:21-62``).

``export_warpgroup_schedule`` keeps the reference's contract: the solve result's lanes
must cover the problem's operations, the schedule with every candidate relation (the
required completion relations with a finite instance) must verify, and each candidate
is then dropped, in sorted order, when every one of its instances stays reachable
through the lanes and the relations still retained. The reachability work runs in the
frame-analysis kernel (``tfv_export_sync``): one closure of the complete set answers
every query, because dropping an edge that another path implies changes no
reachability. Both verifications run on the GPU rows kernel.
"""

from __future__ import annotations

import ctypes
import importlib
from typing import Any, Sequence

import numpy as np

from . import _lib
from .errors import WarpgroupVerificationError
from .verify import _torch, _verifier_for, raise_for_verdict


def _records_module(result: Any):
    """The module that defines the solve result's records (the reference's or the mirror's)."""
    lane_type = type(result.lanes[0]) if result.lanes else type(result)
    return importlib.import_module(lane_type.__module__)


def _check_inputs(problem: Any, result: Any) -> None:
    """sync.py:24-39: exact record types, and lanes that cover the problem's operations."""
    if type(problem).__name__ != "WarpgroupProblem":
        raise WarpgroupVerificationError("export requires an exact WarpgroupProblem")
    if type(result).__name__ != "WarpgroupSolveResult":
        raise WarpgroupVerificationError("export requires an exact WarpgroupSolveResult")
    expected = {operation.id for operation in problem.loop.ops}
    lane_of = {op: index for index, lane in enumerate(result.lanes) for op in lane.operations}
    if len(result.lanes) != problem.warp_groups or set(lane_of) != expected:
        raise WarpgroupVerificationError("solve result lanes do not exactly cover the problem operations")


def export_warpgroup_schedules(problem: Any, results: Sequence[Any], *, device: int = 0) -> list:
    """Export many solve results of one problem in one batch.

    Returns, per result, the exported schedule record or the exception the reference
    would raise for it (the results are independent, so one failure does not stop the
    batch).
    """
    verifier = _verifier_for(problem, device)
    packed = verifier.packed
    iterations = packed.iterations
    candidates = sorted(  # sync.py:41-45, in the order a frame's sync set is stored
        (packed.op_ids[int(a)], packed.op_ids[int(b)], int(d)) for a, b, d in packed.relations if int(d) < iterations
    )
    outcome: list[Any] = [None] * len(results)
    complete, live = [], []
    for k, result in enumerate(results):
        try:
            _check_inputs(problem, result)
        except WarpgroupVerificationError as error:
            outcome[k] = error
            continue
        lanes = [list(lane.operations) for lane in result.lanes]
        rows = [(t.iteration, t.operation_id, t.start, t.issue_end, t.completion) for t in result.times]
        complete.append((lanes, list(candidates), rows))
        live.append(k)
    if not live:
        return outcome
    verdict, _makespan, _ii = verifier.verify_schedules(complete)  # sync.py:46-47

    torch = _torch()
    frames = verifier.new_frames()
    frame_of = [frames.add(lanes, sync) for lanes, sync, _rows in complete]
    dframes = verifier.frames_to_device(frames)
    dev = torch.device("cuda", verifier.device)
    stride = max(1, len(candidates))
    with torch.cuda.device(dev):
        table = torch.empty(verifier.frame_table_bytes(dframes), dtype=torch.uint8, device=dev)
        keep = torch.empty((len(frames), stride), dtype=torch.uint8, device=dev)
        _lib.check(
            verifier._lib.tfv_export_sync(
                verifier._handle, ctypes.byref(dframes.struct), table.data_ptr(), int(table.numel()), keep.data_ptr(),
                stride, verifier._stream(None),
            ),
            "tfv_export_sync",
        )
        mask = keep.cpu().numpy().astype(bool)

    exported, exported_index = [], []
    for j, k in enumerate(live):
        if verdict[j] != 0:
            try:
                raise_for_verdict(int(verdict[j]))
            except Exception as error:  # noqa: BLE001 - handed back per result
                outcome[k] = error
            continue
        records = _records_module(results[k])
        retained = [edge for i, edge in enumerate(candidates) if mask[frame_of[j], i]]
        schedule = records.WarpgroupSchedule(
            records.SCHEDULE_FORMAT,
            results[k].lanes,
            tuple(records.SynchronizationEdge(*edge) for edge in retained),
            results[k].times,
        )
        exported.append(schedule)
        exported_index.append(k)
    if exported:
        final, _m, _i = verifier.verify_schedules(exported)  # sync.py:60-61
        for schedule, k, v in zip(exported, exported_index, final):
            try:
                raise_for_verdict(int(v))
                outcome[k] = schedule
            except Exception as error:  # noqa: BLE001
                outcome[k] = error
    return outcome


def export_warpgroup_schedule(problem: Any, result: Any, *, device: int = 0):
    """Export and transitively reduce the synchronization of one solve result (sync.py:21-62)."""
    (found,) = export_warpgroup_schedules(problem, [result], device=device)
    if isinstance(found, BaseException):
        raise found
    return found


__all__ = ["export_warpgroup_schedule", "export_warpgroup_schedules"]
