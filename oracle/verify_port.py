"""CPU restatement of TileFoundry's warpgroup schedule verifier (test infrastructure only).

This module is the ORACLE: it restates, step for step, the reference verifier
``src/tilefoundry/schedule/warpgroup/verify.py`` together with the schedule
record constructors it depends on (``model.py:425-507``) so that the GPU path
can be checked against it. It is imported only by ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``; no product code path may call it.

Parity pin: ``tests/golden/make_golden.py`` runs the reference itself (in the
build container, where it is importable) on the MLA example and on hand-built
and perturbed schedules, and commits the reference's verdicts as fixtures; the
CPU test suite checks this restatement against every one of them.

Inputs are duck-typed: ``problem`` is any object shaped like the reference's
``WarpgroupProblem`` (``model.py:377``): ``warp_groups``, ``resources``
(``id``, ``capacity``), ``types`` (``id``, ``space``), ``inputs`` (``id``,
``type_id``), ``loop`` with ``iterations``, ``iter_args`` (``id``,
``yield_value.id``) and ``ops`` (``id``, ``warp_group``, ``issue_duration``,
``completion_latency``, ``resource_windows``, ``outputs``). The reference's own
records and the mirror records of ``tilefoundry_b200.model`` both qualify.

A raw candidate is ``(lanes, sync, rows)``: ``lanes`` a sequence of sequences
of operation ids, ``sync`` a sequence of ``(after, before, distance)`` and
``rows`` a sequence of ``(iteration, operation_id, start, issue_end,
completion)``. :func:`classify` returns ``(class_id, makespan, ii)`` with the
class ids of the verdict table below (0 = the schedule verifies).
"""

from __future__ import annotations

import re
from collections import defaultdict, deque

# Verdict classes, numbered in the order in which the reference checks them.
PASS = 0
SCHEDULE_MALFORMED = 1  # model.py:469-477, 437-438, 454-455, 497-504 (record constructors)
LANE_COUNT = 2  # verify.py:211-212
LANE_REPEAT = 3  # verify.py:216-217
LANE_COVERAGE = 4  # verify.py:223-226
OWNERSHIP = 5  # verify.py:227-236
DUP_TIMES = 6  # verify.py:244-245
TIME_COVERAGE = 7  # verify.py:246-252
ISSUE_DURATION = 8  # verify.py:256-257
COMPLETION_LATENCY = 9  # verify.py:258-259
II_NONPOSITIVE = 10  # verify.py:262-264
II_MISMATCH = 11  # verify.py:265-276
LANE_ORDER = 12  # verify.py:278-282
SYNC_UNKNOWN_OP = 13  # verify.py:285-286
SYNC_NO_INSTANCE = 14  # verify.py:287-289
SYNC_INEQUALITY = 15  # verify.py:290-292
REGISTER_CROSSES_LANES = 16  # verify.py:296-304
RELATION_TIMING = 17  # verify.py:311-312
RELATION_NO_PATH = 18  # verify.py:313-314
CARRIED_SHARED_LIFETIME = 19  # verify.py:315-318
RESOURCE_CAPACITY = 20  # verify.py:183-200, 320
CYCLE = 21  # verify.py:163-180, 321-322

CLASS_NAMES = {
    0: "PASS",
    1: "SCHEDULE_MALFORMED",
    2: "LANE_COUNT",
    3: "LANE_REPEAT",
    4: "LANE_COVERAGE",
    5: "OWNERSHIP",
    6: "DUP_TIMES",
    7: "TIME_COVERAGE",
    8: "ISSUE_DURATION",
    9: "COMPLETION_LATENCY",
    10: "II_NONPOSITIVE",
    11: "II_MISMATCH",
    12: "LANE_ORDER",
    13: "SYNC_UNKNOWN_OP",
    14: "SYNC_NO_INSTANCE",
    15: "SYNC_INEQUALITY",
    16: "REGISTER_CROSSES_LANES",
    17: "RELATION_TIMING",
    18: "RELATION_NO_PATH",
    19: "CARRIED_SHARED_LIFETIME",
    20: "RESOURCE_CAPACITY",
    21: "CYCLE",
}


class OracleFailure(Exception):
    """Raised inside the restatement at the first violated check."""

    def __init__(self, class_id: int, message: str) -> None:
        super().__init__(message)
        self.class_id = class_id


def _fail(class_id: int, message: str) -> None:
    raise OracleFailure(class_id, message)


# ---------------------------------------------------------------------------
# Identifier and record-constructor rules (model.py / _identifiers.py)
# ---------------------------------------------------------------------------

# _identifiers.py:9 — a portable caller-defined identifier.
_ID = re.compile(r"[A-Za-z_][A-Za-z0-9_.-]*\Z", re.ASCII)


def _valid_id(value: object) -> bool:
    return type(value) is str and _ID.fullmatch(value) is not None


def _is_int(value: object) -> bool:
    return type(value) is int


def construct(lanes, sync, rows):
    """Restate the schedule record constructors; raise class 1 on any violation.

    Follows ``WarpgroupLane.__post_init__`` (model.py:431-439),
    ``SynchronizationEdge.__post_init__`` (model.py:450-455),
    ``TimedOperation.__post_init__`` (model.py:468-477) and
    ``WarpgroupSchedule.__post_init__`` (model.py:489-507). Returns the
    canonical ``(lanes, sync, times)``: lanes as tuples, sync sorted, times
    sorted (model.py:506-507).
    """
    out_lanes = []
    for lane in lanes:
        ops = tuple(lane)
        for op in ops:
            if not _valid_id(op):
                _fail(SCHEDULE_MALFORMED, "lane operation ID must be an identifier")
        if len(ops) != len(set(ops)):
            _fail(SCHEDULE_MALFORMED, "a lane must not repeat an operation")
        out_lanes.append(ops)
    out_sync = []
    for edge in sync:
        after, before, distance = edge
        if not _valid_id(after) or not _valid_id(before):
            _fail(SCHEDULE_MALFORMED, "sync operation ID must be an identifier")
        if not _is_int(distance) or distance < 0:
            _fail(SCHEDULE_MALFORMED, "sync distance must be a non-negative integer")
        if after == before and distance == 0:
            _fail(SCHEDULE_MALFORMED, "sync must not contain a distance-zero self edge")
        out_sync.append((after, before, distance))
    out_times = []
    for row in rows:
        iteration, op, start, issue_end, completion = row
        if not _is_int(iteration) or iteration < 0:
            _fail(SCHEDULE_MALFORMED, "time iteration must be a non-negative integer")
        if not _valid_id(op):
            _fail(SCHEDULE_MALFORMED, "timed operation ID must be an identifier")
        if not _is_int(start) or start < 0:
            _fail(SCHEDULE_MALFORMED, "time start must be a non-negative integer")
        if not _is_int(issue_end) or issue_end <= 0:
            _fail(SCHEDULE_MALFORMED, "time issue end must be a positive integer")
        if not _is_int(completion) or completion <= 0:
            _fail(SCHEDULE_MALFORMED, "time completion must be a positive integer")
        if issue_end <= start:
            _fail(SCHEDULE_MALFORMED, "time issue end must be greater than start")
        if completion < issue_end:
            _fail(SCHEDULE_MALFORMED, "time completion must be >= issue end")
        out_times.append((iteration, op, start, issue_end, completion))
    if not out_lanes:
        _fail(SCHEDULE_MALFORMED, "schedule must contain at least one lane")
    lane_ops = [op for lane in out_lanes for op in lane]
    if len(lane_ops) != len(set(lane_ops)):
        _fail(SCHEDULE_MALFORMED, "an operation must not appear in more than one lane")
    if len(out_sync) != len(set(out_sync)):
        _fail(SCHEDULE_MALFORMED, "schedule contains duplicate sync edges")
    instances = [(row[0], row[1]) for row in out_times]
    if len(instances) != len(set(instances)):
        _fail(SCHEDULE_MALFORMED, "schedule contains duplicate timed instances")
    return tuple(out_lanes), sorted(out_sync), sorted(out_times)


# ---------------------------------------------------------------------------
# Problem-side semantic tables (verify.py:32-86, model.py:842-861, expression.py:590)
# ---------------------------------------------------------------------------


def value_references(expression) -> tuple[str, ...]:
    """SSA uses of one expression in traversal order (expression.py:590-599, fold order 511-584).

    Dispatches on the record's class name so that the reference's expression
    records and the mirror's ``ValueUses`` node are both accepted.
    """
    kind = type(expression).__name__
    if kind == "ValueRef":
        return (expression.id,)
    if kind == "ScalarLiteral":
        return ()
    if kind == "ValueUses":
        return tuple(expression.ids)
    if kind == "IndexExpression":
        return (expression.source.id,)
    if kind in ("CopyExpression", "CastExpression", "TransposeExpression", "ReduceExpression"):
        return value_references(expression.source)
    if kind == "MatmulExpression":
        return value_references(expression.lhs) + value_references(expression.rhs)
    if kind == "ConcatExpression":
        return tuple(ref for item in expression.values for ref in value_references(item))
    if kind == "SelectExpression":
        return (
            value_references(expression.condition)
            + value_references(expression.when_true)
            + value_references(expression.when_false)
        )
    if kind == "ElementwiseExpression":
        return tuple(ref for item in expression.operands for ref in value_references(item))
    raise TypeError(f"unsupported expression record {kind}")


def _space(value) -> str:
    return value.value if hasattr(value, "value") else str(value)


def semantic_tables(problem):
    """owner[value] -> op, space[value], users[value] -> sorted ops (verify.py:32-52)."""
    types = {item.id: item for item in problem.types}
    owner: dict[str, str] = {}
    spaces = {item.id: _space(types[item.type_id].space) for item in problem.inputs}
    users: dict[str, set[str]] = defaultdict(set)
    for operation in problem.loop.ops:
        for output in operation.outputs:
            owner[output.id] = operation.id
            spaces[output.id] = _space(types[output.type_id].space)
            for value_id in value_references(output.expression):
                users[value_id].add(operation.id)
    for iter_arg in problem.loop.iter_args:
        owner[iter_arg.id] = owner[iter_arg.yield_value.id]
        spaces[iter_arg.id] = spaces[iter_arg.yield_value.id]
    return owner, spaces, {key: tuple(sorted(ops)) for key, ops in users.items()}


def dependencies(problem) -> list[tuple[str, str, int]]:
    """SSA def-use dependencies (model.py:842-861): distance 0 in-body, 1 through iter_args."""
    external = {item.id for item in problem.inputs}
    owner = {out.id: op.id for op in problem.loop.ops for out in op.outputs}
    carried = {item.id: owner[item.yield_value.id] for item in problem.loop.iter_args}
    edges: set[tuple[str, str, int]] = set()
    for operation in problem.loop.ops:
        for output in operation.outputs:
            for use in value_references(output.expression):
                if use in external:
                    continue
                if use in carried:
                    edges.add((carried[use], operation.id, 1))
                    continue
                defining = owner[use]
                if defining != operation.id:
                    edges.add((defining, operation.id, 0))
    return sorted(edges)


def required_completion_relations(problem) -> list[tuple[str, str, int]]:
    """SSA dependencies plus shared-memory WAR edges, sorted (verify.py:55-71)."""
    _owner, spaces, users = semantic_tables(problem)
    relations = set(dependencies(problem))
    for operation in problem.loop.ops:
        for output in operation.outputs:
            if spaces[output.id] != "shared":
                continue
            for user in users.get(output.id, ()):
                if user != operation.id:
                    relations.add((user, operation.id, 1))
    return sorted(relations)


def carried_shared_lifetime_edges(problem) -> set:
    """(i, user) -> (i, defining op) for shared iter_args, i in [1, I) (verify.py:74-86)."""
    owner, spaces, users = semantic_tables(problem)
    edges = set()
    for iter_arg in problem.loop.iter_args:
        if spaces[iter_arg.id] != "shared":
            continue
        defining = owner[iter_arg.id]
        for user in users.get(iter_arg.id, ()):
            if user == defining:
                continue
            for iteration in range(1, problem.loop.iterations):
                edges.add(((iteration, user), (iteration, defining)))
    return edges


# ---------------------------------------------------------------------------
# Instance and event graphs (verify.py:89-180)
# ---------------------------------------------------------------------------


def expand_relation(edge, iterations: int):
    """(i, after) -> (i + d, before) for i < I - d (verify.py:89-96)."""
    after, before, distance = edge
    return tuple(
        ((iteration, after), (iteration + distance, before))
        for iteration in range(max(iterations - distance, 0))
    )


def lane_edges(lanes, iterations: int) -> set:
    """Consecutive lane pairs per iteration plus the wrap edge (verify.py:99-112)."""
    edges = set()
    for lane in lanes:
        for iteration in range(iterations):
            for after, before in zip(lane, lane[1:]):
                edges.add(((iteration, after), (iteration, before)))
            if lane and iteration + 1 < iterations:
                edges.add(((iteration, lane[-1]), (iteration + 1, lane[0])))
    return edges


def control_edges(lanes, sync, iterations: int) -> set:
    """Lane edges plus expanded sync edges (verify.py:115-119)."""
    edges = lane_edges(lanes, iterations)
    for edge in sync:
        edges.update(expand_relation(edge, iterations))
    return edges


def completion_event_edges(problem, lanes, sync) -> set:
    """Unrolled start/issue_end/completion event graph (verify.py:122-141)."""
    iterations = problem.loop.iterations
    edges = set()
    for iteration in range(iterations):
        for operation in problem.loop.ops:
            start = (iteration, operation.id, "start")
            issue_end = (iteration, operation.id, "issue_end")
            completion = (iteration, operation.id, "completion")
            edges.add((start, issue_end))
            edges.add((issue_end, completion))
            if operation.issue_duration == operation.completion_latency:
                edges.add((completion, issue_end))
    for after, before in lane_edges(lanes, iterations):
        edges.add(((*after, "issue_end"), (*before, "start")))
    for edge in sync:
        for after, before in expand_relation(edge, iterations):
            edges.add(((*after, "completion"), (*before, "start")))
    return edges


def event_reachable(edges, source, target) -> bool:
    """DFS from completion(source) to start(target), successor map rebuilt per query (verify.py:144-160)."""
    successors = defaultdict(set)
    for after, before in edges:
        successors[after].add(before)
    source_event = (*source, "completion")
    target_event = (*target, "start")
    pending = [source_event]
    visited = {source_event}
    while pending:
        current = pending.pop()
        if current == target_event:
            return True
        for successor in successors.get(current, ()):
            if successor not in visited:
                visited.add(successor)
                pending.append(successor)
    return False


def require_acyclic(nodes, edges) -> None:
    """Kahn's algorithm over the expanded instance graph (verify.py:163-180)."""
    successors = defaultdict(set)
    indegree = {node: 0 for node in nodes}
    for after, before in edges:
        if before not in successors[after]:
            successors[after].add(before)
            indegree[before] += 1
    ready = deque(sorted(node for node, degree in indegree.items() if degree == 0))
    visited = 0
    while ready:
        current = ready.popleft()
        visited += 1
        for successor in sorted(successors.get(current, ())):
            indegree[successor] -= 1
            if indegree[successor] == 0:
                ready.append(successor)
    if visited != len(nodes):
        _fail(CYCLE, "expanded lane, sync, and semantic graph contains a cycle")


def verify_resources(problem, times) -> None:
    """Netted +amount/-amount sweep per resource in id order (verify.py:183-200)."""
    operations = {item.id: item for item in problem.loop.ops}
    for resource in sorted(problem.resources, key=lambda item: item.id):
        changes = defaultdict(int)
        for instance, timed in times.items():
            operation = operations[instance[1]]
            for window in operation.resource_windows:
                if window.resource_id != resource.id:
                    continue
                start = timed[0]
                end = start + window.duration
                changes[start] += window.amount
                changes[end] -= window.amount
        demand = 0
        for timestamp in sorted(changes):
            demand += changes[timestamp]
            if demand > resource.capacity:
                _fail(RESOURCE_CAPACITY, f"resource {resource.id!r} exceeds capacity at {timestamp}")


# ---------------------------------------------------------------------------
# The ordered check (verify.py:203-322)
# ---------------------------------------------------------------------------


def verify_canonical(problem, lanes, sync, times_rows) -> None:
    """Restate ``_verify_warpgroup_schedule`` (verify.py:203-322); raise at the first failure.

    ``times_rows`` are canonical sorted rows ``(iteration, op, start, issue_end, completion)``.
    """
    iterations = problem.loop.iterations
    operation_by_id = {item.id: item for item in problem.loop.ops}
    expected_operations = set(operation_by_id)
    if len(lanes) != problem.warp_groups:
        _fail(LANE_COUNT, "schedule lane count does not match warp_groups")
    lane_operations = tuple(op for lane in lanes for op in lane)
    if len(lane_operations) != len(set(lane_operations)):
        _fail(LANE_REPEAT, "schedule repeats an operation across lanes")
    lane_by_operation = {op: index for index, lane in enumerate(lanes) for op in lane}
    if set(lane_by_operation) != expected_operations:
        _fail(LANE_COVERAGE, "schedule lane coverage differs")
    for operation in sorted(problem.loop.ops, key=lambda item: item.id):
        if operation.warp_group is None:
            continue
        if lane_by_operation[operation.id] != operation.warp_group:
            _fail(
                OWNERSHIP,
                f"operation {operation.id!r} is scheduled on lane "
                f"{lane_by_operation[operation.id]}, expected warp_group {operation.warp_group}",
            )

    expected_instances = {(i, op) for i in range(iterations) for op in expected_operations}
    times = {(row[0], row[1]): row[2:] for row in times_rows}
    if len(times) != len(times_rows):
        _fail(DUP_TIMES, "schedule contains duplicate timed instances")
    if set(times) != expected_instances:
        _fail(TIME_COVERAGE, "schedule time coverage differs")
    for instance, (start, issue_end, completion) in times.items():
        operation = operation_by_id[instance[1]]
        if issue_end - start != operation.issue_duration:
            _fail(ISSUE_DURATION, f"timed operation {instance!r} has the wrong duration: issue duration")
        if completion - start != operation.completion_latency:
            _fail(
                COMPLETION_LATENCY,
                f"timed operation {instance!r} has the wrong duration: completion latency",
            )
    if iterations >= 3:
        first = min(expected_operations)
        initiation_interval = times[(2, first)][0] - times[(1, first)][0]
        if initiation_interval <= 0:
            _fail(II_NONPOSITIVE, "periodic initiation interval must be positive")
        for op in sorted(expected_operations):
            for iteration in range(1, iterations - 1):
                if times[(iteration + 1, op)][0] - times[(iteration, op)][0] != initiation_interval:
                    _fail(II_MISMATCH, f"periodic initiation interval differs for {op!r}")

    for after, before in lane_edges(lanes, iterations):
        if times[after][1] > times[before][0]:
            _fail(LANE_ORDER, f"lane order {after!r} -> {before!r} is not respected")

    for edge in sync:
        if edge[0] not in expected_operations or edge[1] not in expected_operations:
            _fail(SYNC_UNKNOWN_OP, f"sync edge names an unknown operation: {edge!r}")
        expanded = expand_relation(edge, iterations)
        if not expanded:
            _fail(SYNC_NO_INSTANCE, f"sync edge has no finite instance: {edge!r}")
        for after, before in expanded:
            if times[after][2] > times[before][0]:
                _fail(SYNC_INEQUALITY, f"sync inequality {after!r} -> {before!r} is not respected")

    semantic_edges = set()
    owner, spaces, users = semantic_tables(problem)
    for value_id, space in spaces.items():
        if space != "register":
            continue
        component = set(users.get(value_id, ()))
        if value_id in owner:
            component.add(owner[value_id])
        if len({lane_by_operation[item] for item in component}) > 1:
            _fail(REGISTER_CROSSES_LANES, f"register value {value_id!r} crosses warpgroup lanes")

    controls = control_edges(lanes, sync, iterations)
    completion_edges = completion_event_edges(problem, lanes, sync)
    for relation in required_completion_relations(problem):
        for after, before in expand_relation(relation, iterations):
            semantic_edges.add((after, before))
            if times[after][2] > times[before][0]:
                _fail(RELATION_TIMING, f"completion relation {after!r} -> {before!r} is not respected")
            if not event_reachable(completion_edges, after, before):
                _fail(
                    RELATION_NO_PATH,
                    f"completion relation {after!r} -> {before!r} has no lane/sync path",
                )
    for after, before in carried_shared_lifetime_edges(problem):
        semantic_edges.add((after, before))
        if times[after][2] > times[before][0]:
            _fail(CARRIED_SHARED_LIFETIME, f"carried shared lifetime {after!r} -> {before!r}")

    verify_resources(problem, times)
    require_acyclic(set(expected_instances), controls | semantic_edges)


def makespan_and_ii(problem, rows) -> tuple[int, int]:
    """makespan = max completion (api.py:29-33); II by verify.py:261-262 when I >= 3, else 0."""
    makespan = max((row[4] for row in rows), default=0)
    ii = 0
    if problem.loop.iterations >= 3 and problem.loop.ops:
        first = min(op.id for op in problem.loop.ops)
        starts = {(row[0], row[1]): row[2] for row in rows}
        if (2, first) in starts and (1, first) in starts:
            ii = starts[(2, first)] - starts[(1, first)]
    return makespan, ii


def classify(problem, lanes, sync, rows) -> tuple[int, int, int]:
    """Return ``(class_id, makespan, ii)`` for one raw candidate."""
    makespan, ii = makespan_and_ii(problem, rows)
    try:
        canonical = construct(lanes, sync, rows)
        verify_canonical(problem, *canonical)
    except OracleFailure as failure:
        return failure.class_id, makespan, ii
    return PASS, makespan, ii


def materialize_periodic(problem, prologue: dict, offset: dict, ii: int):
    """Rows of a compact periodic candidate (solve.py:206-231).

    Iteration 0 starts at ``prologue[op]``; iteration i >= 1 at
    ``offset[op] + i * ii``; issue end and completion add the operation's
    issue duration and completion latency.
    """
    rows = []
    for iteration in range(problem.loop.iterations):
        for operation in problem.loop.ops:
            start = prologue[operation.id] if iteration == 0 else offset[operation.id] + iteration * ii
            rows.append(
                (
                    iteration,
                    operation.id,
                    start,
                    start + operation.issue_duration,
                    start + operation.completion_latency,
                )
            )
    return rows


# ---------------------------------------------------------------------------
# Canonical synchronization export (sync.py:21-62)
# ---------------------------------------------------------------------------


def export_sync(problem, lanes, times_rows):
    """Restate ``export_warpgroup_schedule`` (sync.py:21-62) for one solve result.

    ``lanes`` is a tuple of op-id tuples and ``times_rows`` canonical rows. Returns
    ``("ok", retained)`` with the retained relations in candidate order, or
    ``("fail", class_id)`` when the schedule with every candidate relation does not
    verify (sync.py:46-47). The candidates are the required completion relations with a
    finite instance (sync.py:41-45); each is dropped, in order, when every one of its
    instances stays reachable through the lanes and the relations still retained
    (sync.py:49-58).
    """
    iterations = problem.loop.iterations
    candidates = tuple(edge for edge in required_completion_relations(problem) if edge[2] < iterations)
    try:
        verify_canonical(problem, lanes, tuple(sorted(candidates)), times_rows)
    except OracleFailure as failure:
        return "fail", failure.class_id
    retained = list(candidates)
    for candidate in candidates:
        trial = tuple(item for item in retained if item != candidate)
        control = completion_event_edges(problem, lanes, trial)
        if all(event_reachable(control, after, before) for after, before in expand_relation(candidate, iterations)):
            retained.remove(candidate)
    verify_canonical(problem, lanes, tuple(sorted(retained)), times_rows)  # sync.py:60-61
    return "ok", tuple(retained)
