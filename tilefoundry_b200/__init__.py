"""Batched GPU verifier of TileFoundry warpgroup schedules for NVIDIA B200 (sm_100a).

Drop-in for the reference's verification path
(``src/tilefoundry/schedule/warpgroup/verify.py``): the same entry-point names,
arguments and exceptions, with the checks executed by hand-written CUDA kernels in
``libtfv.so`` (C ABI in ``include/tfv.h``), one batch of candidate schedules at a time.
"""

from .errors import (
    VerifierRangeError,
    VerifierRuntimeError,
    WarpgroupSerializationError,
    WarpgroupValidationError,
    WarpgroupVerificationError,
)
from .model import (
    SCHEDULE_FORMAT,
    LoopIterArg,
    MemorySpace,
    OperationOutput,
    ProblemLoop,
    ProblemOperation,
    ProgramInput,
    ResourceCapacity,
    ResourceWindow,
    SynchronizationEdge,
    TensorType,
    TimedOperation,
    ValueRef,
    ValueUses,
    WarpgroupLane,
    WarpgroupProblem,
    WarpgroupSchedule,
    WarpgroupSolveResult,
)
from .problem import PackedProblem, pack_problem
from .serialization import problem_from_json, problem_to_json, schedule_from_json, schedule_to_json
from .sync import export_warpgroup_schedule, export_warpgroup_schedules
from .verify import (
    CLASS_NAMES,
    WarpgroupVerifier,
    _verify_warpgroup_schedule,
    raise_for_verdict,
    verify_warpgroup_schedule,
    verify_warpgroup_schedules,
)

__version__ = "0.1.0"

__all__ = [
    "CLASS_NAMES",
    "LoopIterArg",
    "MemorySpace",
    "OperationOutput",
    "PackedProblem",
    "ProblemLoop",
    "ProblemOperation",
    "ProgramInput",
    "ResourceCapacity",
    "ResourceWindow",
    "SCHEDULE_FORMAT",
    "SynchronizationEdge",
    "WarpgroupSolveResult",
    "export_warpgroup_schedule",
    "export_warpgroup_schedules",
    "TensorType",
    "TimedOperation",
    "ValueRef",
    "ValueUses",
    "VerifierRangeError",
    "VerifierRuntimeError",
    "WarpgroupLane",
    "WarpgroupProblem",
    "WarpgroupSchedule",
    "WarpgroupSerializationError",
    "WarpgroupValidationError",
    "WarpgroupVerificationError",
    "WarpgroupVerifier",
    "_verify_warpgroup_schedule",
    "pack_problem",
    "problem_from_json",
    "problem_to_json",
    "raise_for_verdict",
    "schedule_from_json",
    "schedule_to_json",
    "verify_warpgroup_schedule",
    "verify_warpgroup_schedules",
]
