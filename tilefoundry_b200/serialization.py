"""JSON codecs for the verifier's two input documents.

* The schedule document keeps the reference's format exactly
  (``src/tilefoundry/schedule/warpgroup/serialization.py:679-727`` and
  ``schemas/warpgroup-schedule.schema.json``): an object with exactly
  ``format``, ``lanes``, ``sync`` and ``times``, sync edges as
  ``{"after", "before", "distance"}`` objects and time rows as
  ``[iteration, operation, start, issue_end, completion]``.
* The closed-problem document (format ``tilefoundry_b200.closed_problem``) is
  this package's own: the integer closure that ``build_warpgroup_problem``
  (``build.py:169-220``) produces from a program and hardware document, with
  each output's expression reduced to the SSA values it reads. It lets a
  problem travel without the reference's cost-signature machinery.
"""

from __future__ import annotations

import json

from .errors import WarpgroupSerializationError, WarpgroupValidationError
from .model import (
    PROBLEM_FORMAT,
    LoopIterArg,
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
    value_references,
)


def _pairs(pairs: list[tuple[str, object]]) -> dict[str, object]:
    result: dict[str, object] = {}
    for key, value in pairs:
        if key in result:
            raise WarpgroupSerializationError(f"duplicate JSON field {key!r}")
        result[key] = value
    return result


def _reject_constant(token: str) -> object:
    raise WarpgroupSerializationError(f"non-finite JSON number {token}")


def _loads(text: str) -> object:
    if type(text) is not str:
        raise WarpgroupSerializationError("JSON document must be text")
    try:
        return json.loads(text, object_pairs_hook=_pairs, parse_constant=_reject_constant)
    except WarpgroupSerializationError:
        raise
    except ValueError as error:
        raise WarpgroupSerializationError(f"invalid JSON: {error}") from error


def _object(value: object, fields: frozenset[str], label: str) -> dict[str, object]:
    if type(value) is not dict:
        raise WarpgroupSerializationError(f"{label} must be a JSON object")
    keys = set(value)
    if keys != fields:
        missing = sorted(fields - keys)
        unknown = sorted(keys - fields)
        raise WarpgroupSerializationError(f"{label} fields differ: missing={missing!r}, unknown={unknown!r}")
    return value


def _array(value: object, label: str) -> list[object]:
    if type(value) is not list:
        raise WarpgroupSerializationError(f"{label} must be a JSON array")
    return value


def _integer(value: object, label: str) -> int:
    if type(value) is not int:
        raise WarpgroupSerializationError(f"{label} must be an integer")
    return value


def _string(value: object, label: str) -> str:
    if type(value) is not str:
        raise WarpgroupSerializationError(f"{label} must be a string")
    return value


# --------------------------------------------------------------------------- schedule


def schedule_from_json(text: str) -> WarpgroupSchedule:
    """Decode one strict schedule document into validated records."""
    try:
        data = _object(_loads(text), frozenset({"format", "lanes", "sync", "times"}), "warpgroup schedule")
        lanes = tuple(
            WarpgroupLane(tuple(_string(item, "lane operation") for item in _array(raw, "lane")))
            for raw in _array(data["lanes"], "lanes")
        )
        sync = []
        for raw in _array(data["sync"], "sync"):
            item = _object(raw, frozenset({"after", "before", "distance"}), "sync edge")
            sync.append(
                SynchronizationEdge(
                    _string(item["after"], "sync after"),
                    _string(item["before"], "sync before"),
                    _integer(item["distance"], "sync distance"),
                )
            )
        times = []
        for raw in _array(data["times"], "times"):
            row = _array(raw, "time row")
            if len(row) != 5:
                raise WarpgroupSerializationError("time row must contain exactly 5 items")
            times.append(
                TimedOperation(
                    _integer(row[0], "time iteration"),
                    _string(row[1], "timed operation ID"),
                    _integer(row[2], "time start"),
                    _integer(row[3], "time issue end"),
                    _integer(row[4], "time completion"),
                )
            )
        return WarpgroupSchedule(_string(data["format"], "schedule format"), lanes, tuple(sync), tuple(times))
    except WarpgroupSerializationError:
        raise
    except WarpgroupValidationError as error:
        raise WarpgroupSerializationError(str(error)) from error


def schedule_to_json(schedule: WarpgroupSchedule) -> str:
    """Canonical JSON for one schedule (sorted sync and times, compact separators)."""
    payload = {
        "format": schedule.format,
        "lanes": [list(lane.operations) for lane in schedule.lanes],
        "sync": [{"after": e.after, "before": e.before, "distance": e.distance} for e in schedule.sync],
        "times": [[t.iteration, t.operation_id, t.start, t.issue_end, t.completion] for t in schedule.times],
    }
    return json.dumps(payload, sort_keys=True, separators=(",", ":"))


# --------------------------------------------------------------------------- closed problem


def problem_from_json(text: str) -> WarpgroupProblem:
    """Decode a closed-problem document."""
    try:
        data = _object(
            _loads(text),
            frozenset({"format", "time_unit", "warp_groups", "resources", "types", "inputs", "loop"}),
            "closed problem",
        )
        if data["format"] != PROBLEM_FORMAT:
            raise WarpgroupSerializationError(f"problem format must be {PROBLEM_FORMAT!r}")
        resources = tuple(
            ResourceCapacity(
                _string(item["id"], "resource id"), _integer(item["capacity"], "resource capacity")
            )
            for item in (_object(raw, frozenset({"id", "capacity"}), "resource") for raw in _array(data["resources"], "resources"))
        )
        types = tuple(
            TensorType(_string(item["id"], "type id"), _string(item["space"], "type space"))
            for item in (_object(raw, frozenset({"id", "space"}), "type") for raw in _array(data["types"], "types"))
        )
        inputs = tuple(
            ProgramInput(_string(item["id"], "input id"), _string(item["type_id"], "input type"))
            for item in (_object(raw, frozenset({"id", "type_id"}), "input") for raw in _array(data["inputs"], "inputs"))
        )
        loop = _object(data["loop"], frozenset({"index", "iterations", "iter_args", "ops"}), "loop")
        iter_args = tuple(
            LoopIterArg(_string(item["id"], "iter_arg id"), ValueRef(_string(item["yield"], "iter_arg yield")))
            for item in (_object(raw, frozenset({"id", "yield"}), "iter_arg") for raw in _array(loop["iter_args"], "iter_args"))
        )
        ops = []
        for raw in _array(loop["ops"], "ops"):
            item = _object(
                raw,
                frozenset({"id", "warp_group", "issue_duration", "completion_latency", "resource_windows", "outputs"}),
                "operation",
            )
            warp_group = item["warp_group"]
            if warp_group is not None:
                warp_group = _integer(warp_group, "warp_group")
            windows = []
            for window in _array(item["resource_windows"], "resource windows"):
                triple = _array(window, "resource window")
                if len(triple) != 3:
                    raise WarpgroupSerializationError("resource window must be [resource, amount, duration]")
                windows.append(
                    ResourceWindow(
                        _string(triple[0], "window resource"),
                        _integer(triple[1], "window amount"),
                        _integer(triple[2], "window duration"),
                    )
                )
            outputs = tuple(
                OperationOutput(
                    _string(out["id"], "output id"),
                    _string(out["type_id"], "output type"),
                    ValueUses(tuple(_string(use, "use") for use in _array(out["uses"], "uses"))),
                )
                for out in (_object(o, frozenset({"id", "type_id", "uses"}), "output") for o in _array(item["outputs"], "outputs"))
            )
            ops.append(
                ProblemOperation(
                    _string(item["id"], "operation id"),
                    outputs,
                    warp_group,
                    _integer(item["issue_duration"], "issue duration"),
                    _integer(item["completion_latency"], "completion latency"),
                    tuple(windows),
                )
            )
        return WarpgroupProblem(
            _string(data["time_unit"], "time_unit"),
            _integer(data["warp_groups"], "warp_groups"),
            resources,
            types,
            inputs,
            ProblemLoop(
                _string(loop["index"], "loop index"),
                _integer(loop["iterations"], "iterations"),
                iter_args,
                tuple(ops),
            ),
        )
    except WarpgroupSerializationError:
        raise
    except (WarpgroupValidationError, KeyError, TypeError) as error:
        raise WarpgroupSerializationError(str(error)) from error


def problem_to_json(problem: object) -> str:
    """Encode any problem shaped like ``WarpgroupProblem`` (the reference's included)."""

    def space(value: object) -> str:
        return value.value if hasattr(value, "value") else str(value)  # type: ignore[attr-defined]

    payload = {
        "format": PROBLEM_FORMAT,
        "time_unit": problem.time_unit,  # type: ignore[attr-defined]
        "warp_groups": problem.warp_groups,  # type: ignore[attr-defined]
        "resources": [{"id": r.id, "capacity": r.capacity} for r in problem.resources],  # type: ignore[attr-defined]
        "types": [{"id": t.id, "space": space(t.space)} for t in problem.types],  # type: ignore[attr-defined]
        "inputs": [{"id": i.id, "type_id": i.type_id} for i in problem.inputs],  # type: ignore[attr-defined]
        "loop": {
            "index": problem.loop.index,  # type: ignore[attr-defined]
            "iterations": problem.loop.iterations,  # type: ignore[attr-defined]
            "iter_args": [{"id": a.id, "yield": a.yield_value.id} for a in problem.loop.iter_args],  # type: ignore[attr-defined]
            "ops": [
                {
                    "id": op.id,
                    "warp_group": op.warp_group,
                    "issue_duration": op.issue_duration,
                    "completion_latency": op.completion_latency,
                    "resource_windows": [[w.resource_id, w.amount, w.duration] for w in op.resource_windows],
                    "outputs": [
                        {"id": o.id, "type_id": o.type_id, "uses": list(value_references(o.expression))}
                        for o in op.outputs
                    ],
                }
                for op in problem.loop.ops  # type: ignore[attr-defined]
            ],
        },
    }
    return json.dumps(payload, sort_keys=True, separators=(",", ":"))


__all__ = ["problem_from_json", "problem_to_json", "schedule_from_json", "schedule_to_json"]
