"""Immutable records consumed by the batched verifier.

These mirror the reference records that the verification path reads
(``src/tilefoundry/schedule/warpgroup/model.py``): the closed problem
(``WarpgroupProblem`` :377, ``ProblemLoop`` :312, ``ProblemOperation`` :248,
``ResourceCapacity`` :222, ``ResourceWindow`` :234) and the schedule
(``WarpgroupSchedule`` :481, ``WarpgroupLane`` :426, ``SynchronizationEdge``
:443, ``TimedOperation`` :459). Field names, canonical sort orders and the
schedule constructors' validation rules are kept identical because the
verifier's verdict depends on them: a schedule that the reference refuses to
construct is verdict class 1 here too.

The packer accepts the reference's own records as well (it reads attributes
only), so a caller that already holds a reference ``WarpgroupProblem`` can
pass it unchanged.

Expressions: the verifier needs only the SSA values an output reads. The
closed-problem document therefore stores each output's uses as a
:class:`ValueUses` node (ids in traversal order); the reference's full
expression records are accepted too (see :func:`value_references`).
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from enum import Enum

from .errors import WarpgroupValidationError

SCHEDULE_FORMAT = "tilefoundry.warpgroup_schedule"
PROBLEM_FORMAT = "tilefoundry_b200.closed_problem"

# Identifier grammar of _identifiers.py:9-10.
_ID = re.compile(r"[A-Za-z_][A-Za-z0-9_.-]*\Z", re.ASCII)
_SSA_ID = re.compile(r"%[A-Za-z_][A-Za-z0-9_.-]*\Z", re.ASCII)


def is_identifier(value: object) -> bool:
    """True for a non-empty portable ASCII identifier."""
    return type(value) is str and _ID.fullmatch(value) is not None


def _require_id(value: object, label: str) -> None:
    if not is_identifier(value):
        raise WarpgroupValidationError(f"{label} must be a non-empty ASCII identifier, got {value!r}")


def _require_ssa_id(value: object, label: str) -> None:
    if type(value) is not str or _SSA_ID.fullmatch(value) is None:
        raise WarpgroupValidationError(
            f"{label} must be an ASCII SSA identifier beginning with '%', got {value!r}"
        )


def _positive(value: object, label: str) -> None:
    if type(value) is not int or value <= 0:
        raise WarpgroupValidationError(f"{label} must be a positive integer, got {value!r}")


def _non_negative(value: object, label: str) -> None:
    if type(value) is not int or value < 0:
        raise WarpgroupValidationError(f"{label} must be a non-negative integer, got {value!r}")


class MemorySpace(str, Enum):
    """Storage semantics visible to scheduling (model.py:39-44)."""

    REGISTER = "register"
    SHARED = "shared"
    GLOBAL = "global"


@dataclass(frozen=True, slots=True)
class TensorType:
    """A named value type; the verifier reads only its memory space."""

    id: str
    space: MemorySpace
    shape: tuple[int, ...] = ()
    dtype: str | None = None

    def __post_init__(self) -> None:
        _require_id(self.id, "type ID")
        object.__setattr__(self, "space", MemorySpace(self.space))
        object.__setattr__(self, "shape", tuple(self.shape))


@dataclass(frozen=True, slots=True)
class ProgramInput:
    """One external SSA value available at the loop boundary."""

    id: str
    type_id: str

    def __post_init__(self) -> None:
        _require_ssa_id(self.id, "input ID")
        _require_id(self.type_id, "input type ID")


@dataclass(frozen=True, slots=True)
class ValueRef:
    """One use of an SSA value."""

    id: str

    def __post_init__(self) -> None:
        _require_ssa_id(self.id, "value reference")


@dataclass(frozen=True, slots=True)
class ValueUses:
    """The SSA values one output expression reads, in traversal order."""

    ids: tuple[str, ...]

    def __post_init__(self) -> None:
        ids = tuple(self.ids)
        for item in ids:
            _require_ssa_id(item, "value use")
        object.__setattr__(self, "ids", ids)


@dataclass(frozen=True, slots=True)
class LoopIterArg:
    """One loop phi: the value yielded by the body becomes ``id`` next iteration."""

    id: str
    yield_value: ValueRef

    def __post_init__(self) -> None:
        _require_ssa_id(self.id, "iter_arg ID")
        if type(self.yield_value).__name__ != "ValueRef":
            raise WarpgroupValidationError(f"iter_arg {self.id!r} yield must be a ValueRef")


@dataclass(frozen=True, slots=True)
class OperationOutput:
    """One typed SSA definition of an operation."""

    id: str
    type_id: str
    expression: object

    def __post_init__(self) -> None:
        _require_ssa_id(self.id, "operation output ID")
        _require_id(self.type_id, "output type ID")


@dataclass(frozen=True, slots=True)
class ResourceCapacity:
    """One positive temporal-resource capacity (model.py:222)."""

    id: str
    capacity: int

    def __post_init__(self) -> None:
        _require_id(self.id, "resource ID")
        _positive(self.capacity, f"resource {self.id!r} capacity")


@dataclass(frozen=True, slots=True, order=True)
class ResourceWindow:
    """A window of ``amount`` units held for ``duration`` from operation start (model.py:234)."""

    resource_id: str
    amount: int
    duration: int

    def __post_init__(self) -> None:
        _require_id(self.resource_id, "resource window ID")
        _positive(self.amount, "resource window amount")
        _positive(self.duration, "resource window duration")


@dataclass(frozen=True, slots=True)
class ProblemOperation:
    """One operation closed to issue/completion timing and resource windows (model.py:248)."""

    id: str
    outputs: tuple[OperationOutput, ...]
    warp_group: int | None
    issue_duration: int
    completion_latency: int
    resource_windows: tuple[ResourceWindow, ...] = ()

    def __post_init__(self) -> None:
        _require_id(self.id, "operation ID")
        outputs = tuple(self.outputs)
        if not outputs:
            raise WarpgroupValidationError(f"operation {self.id!r} must define an output")
        if self.warp_group is not None:
            _non_negative(self.warp_group, "operation warp_group")
        _positive(self.issue_duration, f"operation {self.id!r} issue duration")
        _positive(self.completion_latency, f"operation {self.id!r} completion latency")
        if self.completion_latency < self.issue_duration:
            raise WarpgroupValidationError(
                f"operation {self.id!r} completion latency must be >= issue duration"
            )
        windows = tuple(self.resource_windows)
        for window in windows:
            if window.duration > self.completion_latency:
                raise WarpgroupValidationError(
                    f"operation {self.id!r} resource window exceeds completion latency"
                )
        object.__setattr__(self, "outputs", tuple(sorted(outputs, key=lambda item: item.id)))
        object.__setattr__(self, "resource_windows", tuple(sorted(windows)))


@dataclass(frozen=True, slots=True)
class ProblemLoop:
    """The finite loop: iteration count, loop-carried values and operations sorted by id."""

    index: str
    iterations: int
    iter_args: tuple[LoopIterArg, ...]
    ops: tuple[ProblemOperation, ...]

    def __post_init__(self) -> None:
        _positive(self.iterations, "loop iterations")
        ops = tuple(self.ops)
        if not ops:
            raise WarpgroupValidationError("loop must contain at least one operation")
        ids = [item.id for item in ops]
        if len(ids) != len(set(ids)):
            raise WarpgroupValidationError("duplicate operation IDs")
        object.__setattr__(self, "iter_args", tuple(sorted(self.iter_args, key=lambda item: item.id)))
        object.__setattr__(self, "ops", tuple(sorted(ops, key=lambda item: item.id)))


@dataclass(frozen=True, slots=True)
class WarpgroupProblem:
    """The pure-integer closure of a program and hardware description (model.py:377)."""

    time_unit: str
    warp_groups: int
    resources: tuple[ResourceCapacity, ...]
    types: tuple[TensorType, ...]
    inputs: tuple[ProgramInput, ...]
    loop: ProblemLoop

    def __post_init__(self) -> None:
        _require_id(self.time_unit, "time_unit")
        _positive(self.warp_groups, "warp_groups")
        resources = tuple(sorted(self.resources, key=lambda item: item.id))
        if len({item.id for item in resources}) != len(resources):
            raise WarpgroupValidationError("duplicate resource IDs")
        object.__setattr__(self, "resources", resources)
        object.__setattr__(self, "types", tuple(sorted(self.types, key=lambda item: item.id)))
        object.__setattr__(self, "inputs", tuple(sorted(self.inputs, key=lambda item: item.id)))
        capacity = {item.id: item.capacity for item in resources}
        for operation in self.loop.ops:
            if operation.warp_group is not None and operation.warp_group >= self.warp_groups:
                raise WarpgroupValidationError(
                    f"problem operation {operation.id!r} warp_group is out of range"
                )
            for window in operation.resource_windows:
                if window.resource_id not in capacity:
                    raise WarpgroupValidationError(
                        f"operation {operation.id!r} uses undefined resource {window.resource_id!r}"
                    )
                if window.amount > capacity[window.resource_id]:
                    raise WarpgroupValidationError(
                        f"operation {operation.id!r} window for {window.resource_id!r} exceeds capacity"
                    )


@dataclass(frozen=True, slots=True)
class WarpgroupLane:
    """The ordered body program of one warpgroup (model.py:426-439)."""

    operations: tuple[str, ...]

    def __post_init__(self) -> None:
        if not isinstance(self.operations, (tuple, list)):
            raise WarpgroupValidationError("lane operations must be a sequence")
        operations = tuple(self.operations)
        for operation in operations:
            _require_id(operation, "lane operation ID")
        if len(operations) != len(set(operations)):
            raise WarpgroupValidationError("a lane must not repeat an operation")
        object.__setattr__(self, "operations", operations)


@dataclass(frozen=True, slots=True, order=True)
class SynchronizationEdge:
    """One completion-to-start happens-before relation (model.py:443-455)."""

    after: str
    before: str
    distance: int

    def __post_init__(self) -> None:
        _require_id(self.after, "sync after operation")
        _require_id(self.before, "sync before operation")
        _non_negative(self.distance, "sync distance")
        if self.after == self.before and self.distance == 0:
            raise WarpgroupValidationError("sync must not contain a distance-zero self edge")


@dataclass(frozen=True, slots=True, order=True)
class TimedOperation:
    """One operation instance with issue end and completion timestamps (model.py:459-477)."""

    iteration: int
    operation_id: str
    start: int
    issue_end: int
    completion: int

    def __post_init__(self) -> None:
        _non_negative(self.iteration, "time iteration")
        _require_id(self.operation_id, "timed operation ID")
        _non_negative(self.start, "time start")
        _positive(self.issue_end, "time issue end")
        _positive(self.completion, "time completion")
        if self.issue_end <= self.start:
            raise WarpgroupValidationError("time issue end must be greater than start")
        if self.completion < self.issue_end:
            raise WarpgroupValidationError("time completion must be >= issue end")


@dataclass(frozen=True, slots=True)
class WarpgroupSchedule:
    """Lane order, synchronization and a concrete timing witness (model.py:481-507)."""

    format: str
    lanes: tuple[WarpgroupLane, ...]
    sync: tuple[SynchronizationEdge, ...]
    times: tuple[TimedOperation, ...]

    def __post_init__(self) -> None:
        if self.format != SCHEDULE_FORMAT:
            raise WarpgroupValidationError(f"schedule format must be {SCHEDULE_FORMAT!r}")
        lanes = tuple(self.lanes)
        sync = tuple(self.sync)
        times = tuple(self.times)
        if not all(type(item) is WarpgroupLane for item in lanes):
            raise WarpgroupValidationError("schedule lanes must contain only exact WarpgroupLane records")
        if not all(type(item) is SynchronizationEdge for item in sync):
            raise WarpgroupValidationError("schedule sync must contain only exact SynchronizationEdge records")
        if not all(type(item) is TimedOperation for item in times):
            raise WarpgroupValidationError("schedule times must contain only exact TimedOperation records")
        if not lanes:
            raise WarpgroupValidationError("schedule must contain at least one lane")
        lane_ops = tuple(op for lane in lanes for op in lane.operations)
        if len(lane_ops) != len(set(lane_ops)):
            raise WarpgroupValidationError("an operation must not appear in more than one lane")
        if len(sync) != len(set(sync)):
            raise WarpgroupValidationError("schedule contains duplicate sync edges")
        instances = tuple((item.iteration, item.operation_id) for item in times)
        if len(instances) != len(set(instances)):
            raise WarpgroupValidationError("schedule contains duplicate timed instances")
        object.__setattr__(self, "lanes", lanes)
        object.__setattr__(self, "sync", tuple(sorted(sync)))
        object.__setattr__(self, "times", tuple(sorted(times)))


@dataclass(frozen=True, slots=True)
class WarpgroupSolveResult:
    """A solver's lane program and timing witness (solve.py:33-60)."""

    status: str
    lanes: tuple[WarpgroupLane, ...]
    times: tuple[TimedOperation, ...]
    initiation_interval: int | None = None

    def __post_init__(self) -> None:
        if self.status not in ("OPTIMAL", "FEASIBLE_NOT_PROVEN"):
            raise WarpgroupValidationError(f"invalid warpgroup solve status {self.status!r}")
        if type(self.lanes) is not tuple or not all(type(item) is WarpgroupLane for item in self.lanes):
            raise WarpgroupValidationError("solve lanes must contain exact WarpgroupLane records")
        if type(self.times) is not tuple or not all(type(item) is TimedOperation for item in self.times):
            raise WarpgroupValidationError("solve times must contain exact TimedOperation records")
        if self.initiation_interval is not None and (
            type(self.initiation_interval) is not int or self.initiation_interval <= 0
        ):
            raise WarpgroupValidationError("initiation interval must be a positive integer")

    @property
    def makespan(self) -> int:
        """The finite makespan of the timing witness."""
        return max((item.completion for item in self.times), default=0)


def value_references(expression: object) -> tuple[str, ...]:
    """SSA values read by one expression, in traversal order.

    Accepts :class:`ValueUses`/:class:`ValueRef` and the reference's expression
    records (``expression.py:590-599``), dispatching on the record's class name.
    """
    kind = type(expression).__name__
    if kind == "ValueRef":
        return (expression.id,)  # type: ignore[attr-defined]
    if kind == "ValueUses":
        return tuple(expression.ids)  # type: ignore[attr-defined]
    if kind == "ScalarLiteral":
        return ()
    if kind == "IndexExpression":
        return (expression.source.id,)  # type: ignore[attr-defined]
    if kind in ("CopyExpression", "CastExpression", "TransposeExpression", "ReduceExpression"):
        return value_references(expression.source)  # type: ignore[attr-defined]
    if kind == "MatmulExpression":
        return value_references(expression.lhs) + value_references(expression.rhs)  # type: ignore[attr-defined]
    if kind == "ConcatExpression":
        return tuple(r for item in expression.values for r in value_references(item))  # type: ignore[attr-defined]
    if kind == "SelectExpression":
        return (
            value_references(expression.condition)  # type: ignore[attr-defined]
            + value_references(expression.when_true)  # type: ignore[attr-defined]
            + value_references(expression.when_false)  # type: ignore[attr-defined]
        )
    if kind == "ElementwiseExpression":
        return tuple(r for item in expression.operands for r in value_references(item))  # type: ignore[attr-defined]
    raise WarpgroupValidationError(f"unsupported expression record {kind}")


__all__ = [
    "LoopIterArg",
    "MemorySpace",
    "OperationOutput",
    "PROBLEM_FORMAT",
    "ProblemLoop",
    "ProblemOperation",
    "ProgramInput",
    "ResourceCapacity",
    "ResourceWindow",
    "SCHEDULE_FORMAT",
    "WarpgroupSolveResult",
    "SynchronizationEdge",
    "TensorType",
    "TimedOperation",
    "ValueRef",
    "ValueUses",
    "WarpgroupLane",
    "WarpgroupProblem",
    "WarpgroupSchedule",
    "is_identifier",
    "value_references",
]
