"""ctypes binding of ``libtfv.so`` (the C ABI declared in ``include/tfv.h``).

The library is loaded from this package directory. There is no fallback: if it is
missing or fails to load, every verifier entry point raises
:class:`~tilefoundry_b200.errors.VerifierRuntimeError`.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

from .errors import VerifierRuntimeError

LIBRARY = Path(__file__).resolve().parent / "libtfv.so"

# Status codes and constants of include/tfv.h.
TFV_OK = 0
TFV_FRAME_MALFORMED = 1
TFV_FRAME_UNKNOWN_LANE_OP = 2
TFV_ROWS_MALFORMED = 1
TFV_ROWS_COVERAGE = 2
TFV_LANE_SHIFT = 12
TFV_LANE_ABSENT = 15
TFV_MAX_LANES = 15
TFV_MAX_OPS = 4095
TFV_TIME_LIMIT = 1 << 30
TFV_BASE_LIMIT = 1 << 28
ABI_VERSION = 5
PLAN_AUTO = 0
PLAN_TILES = 1
PLAN_RING = 2
CLASS_OUT_OF_RANGE = -1
CLASS_BAD_PACKING = -2
CLASS_DEVICE_TIMEOUT = -3


_p = ctypes.c_void_p


class ProblemDesc(ctypes.Structure):
    _fields_ = [
        ("n_ops", ctypes.c_int32),
        ("iterations", ctypes.c_int32),
        ("warp_groups", ctypes.c_int32),
        ("issue_duration", _p),
        ("completion_latency", _p),
        ("warp_group", _p),
        ("n_relations", ctypes.c_int32),
        ("relation_after", _p),
        ("relation_before", _p),
        ("relation_distance", _p),
        ("n_carried", ctypes.c_int32),
        ("carried_user", _p),
        ("carried_def", _p),
        ("n_register_groups", ctypes.c_int32),
        ("register_group_offsets", _p),
        ("register_group_ops", _p),
        ("n_resources", ctypes.c_int32),
        ("resource_capacity", _p),
        ("window_offsets", _p),
        ("window_resource", _p),
        ("window_amount", _p),
        ("window_duration", _p),
    ]


class Frames(ctypes.Structure):
    _fields_ = [
        ("n_frames", ctypes.c_int32),
        ("lane_pos", _p),
        ("lane_count", _p),
        ("flags", _p),
        ("sync_set", _p),
        ("n_sync_sets", ctypes.c_int32),
        ("n_sync_edges", ctypes.c_int32),
        ("sync_offsets", _p),
        ("sync_edges", _p),
    ]


class PlanOptions(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_int32), ("ring_warps", ctypes.c_int32), ("no_delta", ctypes.c_int32)]


class PeriodicBatch(ctypes.Structure):
    _fields_ = [
        ("n_candidates", ctypes.c_int64),
        ("op_stride", ctypes.c_int64),
        ("base_prologue", _p),
        ("base_offset", _p),
        ("prologue_delta", _p),
        ("offset_delta", _p),
        ("ii", _p),
        ("frame", _p),
    ]


class RowsBatch(ctypes.Structure):
    _fields_ = [
        ("n_candidates", ctypes.c_int64),
        ("start", _p),
        ("issue_end", _p),
        ("completion", _p),
        ("frame", _p),
        ("row_flags", _p),
    ]


class Results(ctypes.Structure):
    _fields_ = [("verdict", _p), ("makespan", _p), ("ii", _p)]


def frames_struct(arrays: dict, n_frames: int, pointer=lambda a: a.ctypes.data) -> "Frames":
    """A ``tfv_frames`` over the arrays of :meth:`FrameSet.arrays` (host or device)."""
    return Frames(
        n_frames,
        pointer(arrays["lane_pos"]) if n_frames else None,
        pointer(arrays["lane_count"]) if n_frames else None,
        pointer(arrays["flags"]) if n_frames else None,
        pointer(arrays["sync_set"]) if n_frames else None,
        len(arrays["sync_offsets"]) - 1,
        int(arrays["sync_offsets"][-1]),
        pointer(arrays["sync_offsets"]),
        pointer(arrays["sync_edges"]),
    )


EXPORTS = {
    "tfv_abi_version": (ctypes.c_int, []),
    "tfv_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
    "tfv_set_device_wait_limit": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    "tfv_problem_create": (ctypes.c_int, [ctypes.POINTER(ProblemDesc), ctypes.c_int, ctypes.POINTER(_p)]),
    "tfv_problem_destroy": (ctypes.c_int, [_p]),
    "tfv_frame_table_bytes": (ctypes.c_int, [_p, ctypes.POINTER(Frames), ctypes.POINTER(ctypes.c_size_t)]),
    "tfv_analyze_frames": (ctypes.c_int, [_p, ctypes.POINTER(Frames), _p, ctypes.c_size_t, _p]),
    "tfv_verify_periodic": (
        ctypes.c_int,
        [_p, ctypes.POINTER(Frames), _p, ctypes.c_size_t, ctypes.POINTER(PeriodicBatch), ctypes.POINTER(Results), _p],
    ),
    "tfv_frameset_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_p)]),
    "tfv_frameset_destroy": (ctypes.c_int, [_p]),
    "tfv_frameset_view": (ctypes.c_int, [_p, ctypes.POINTER(Frames)]),
    "tfv_decode_schedules": (
        ctypes.c_int,
        [_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_size_t)] + [_p] * 8 + [ctypes.c_int],
    ),
    "tfv_plan_create": (ctypes.c_int, [_p, ctypes.POINTER(Frames), ctypes.c_int, ctypes.POINTER(_p)]),
    "tfv_plan_create_with": (
        ctypes.c_int, [_p, ctypes.POINTER(Frames), ctypes.c_int, ctypes.POINTER(PlanOptions), ctypes.POINTER(_p)]
    ),
    "tfv_plan_kernel": (ctypes.c_int, [_p]),
    "tfv_plan_delta": (ctypes.c_int, [_p]),
    "tfv_plan_ring_warps": (ctypes.c_int, [_p]),
    "tfv_plan_set_timing": (ctypes.c_int, [_p, ctypes.c_int]),
    "tfv_plan_kernel_times": (ctypes.c_int, [_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "tfv_plan_destroy": (ctypes.c_int, [_p]),
    "tfv_plan_source": (ctypes.c_int, [_p, ctypes.c_char_p, ctypes.c_size_t]),
    "tfv_verify_periodic_planned": (
        ctypes.c_int,
        [_p, ctypes.POINTER(Frames), _p, ctypes.c_size_t, ctypes.POINTER(PeriodicBatch), ctypes.c_int,
         ctypes.POINTER(Results), _p],
    ),
    "tfv_export_sync": (ctypes.c_int, [_p, ctypes.POINTER(Frames), _p, ctypes.c_size_t, _p, ctypes.c_int, _p]),
    "tfv_verify_periodic_sweep": (
        ctypes.c_int,
        [_p, ctypes.POINTER(Frames), _p, ctypes.c_size_t, ctypes.POINTER(PeriodicBatch), ctypes.c_int, _p,
         ctypes.POINTER(Results), _p],
    ),
    "tfv_verify_rows": (
        ctypes.c_int,
        [_p, ctypes.POINTER(Frames), _p, ctypes.POINTER(RowsBatch), ctypes.POINTER(Results), _p],
    ),
    "tfv_verify_periodic_host": (
        ctypes.c_int,
        [_p, ctypes.POINTER(Frames), ctypes.POINTER(PeriodicBatch), ctypes.POINTER(Results)],
    ),
    "tfv_verify_periodic_static": (
        ctypes.c_int,
        [_p, ctypes.POINTER(Frames), ctypes.POINTER(PeriodicBatch), ctypes.POINTER(Results), _p],
    ),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load ``libtfv.so`` once and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise VerifierRuntimeError(
            f"native verifier library missing: {LIBRARY} (build it with `python -m tilefoundry_b200._build`)"
        )
    try:
        lib = ctypes.CDLL(str(LIBRARY))
    except OSError as error:
        raise VerifierRuntimeError(f"cannot load {LIBRARY}: {error}") from error
    for name, (restype, argtypes) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.tfv_abi_version() != ABI_VERSION:
        raise VerifierRuntimeError("libtfv.so ABI version mismatch")
    _lib = lib
    return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().tfv_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    if status != TFV_OK:
        raise VerifierRuntimeError(f"{what} failed with status {status}: {last_error()}")


__all__ = [
    "ABI_VERSION",
    "EXPORTS",
    "frames_struct",
    "Frames",
    "PeriodicBatch",
    "ProblemDesc",
    "Results",
    "RowsBatch",
    "check",
    "last_error",
    "load",
]
