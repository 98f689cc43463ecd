"""Lower a closed warpgroup problem to the integer tables of ``tfv_problem_desc``.

Everything the reference verifier derives from the problem on every call is derived
here once (``src/tilefoundry/schedule/warpgroup/verify.py:32-86`` and
``model.py:842-861``):

* operations in id order (the order ``ProblemLoop`` sorts them into, model.py:330),
  with issue duration, completion latency and declared warp group;
* the required completion relations — SSA def-use dependencies at distance 0 (in-body)
  or 1 (through a loop iter_arg) plus, for every shared-memory output, a distance-1
  relation from each of its users back to its producer (the write-after-read reuse of
  the same allocation) — sorted like ``SynchronizationEdge``;
* the carried shared-lifetime pairs: for a shared iter_arg, each user must complete
  before the yielding operation starts in the same iteration (iterations 1..I-1);
* register groups: the producer and users of every register value, which must share a
  lane;
* resources in id order and each operation's resource windows.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from .errors import WarpgroupValidationError
from .model import value_references

_SPACE_REGISTER = "register"
_SPACE_SHARED = "shared"


def _space(value: object) -> str:
    return value.value if hasattr(value, "value") else str(value)  # type: ignore[attr-defined]


@dataclass
class PackedProblem:
    """Integer tables of one problem (host numpy arrays) plus the id -> index map."""

    op_ids: tuple[str, ...]
    index: dict[str, int]
    iterations: int
    warp_groups: int
    issue: np.ndarray
    latency: np.ndarray
    warp_group: np.ndarray
    relations: np.ndarray  # [R, 3] after, before, distance
    carried: np.ndarray  # [C, 2] user, def
    register_offsets: np.ndarray
    register_ops: np.ndarray
    resource_ids: tuple[str, ...]
    capacity: np.ndarray
    window_offsets: np.ndarray
    window_resource: np.ndarray
    window_amount: np.ndarray
    window_duration: np.ndarray
    _keep: list = field(default_factory=list, repr=False)

    @property
    def n_ops(self) -> int:
        return len(self.op_ids)

    def relation_ids(self) -> list[tuple[str, str, int]]:
        return [(self.op_ids[a], self.op_ids[b], int(d)) for a, b, d in self.relations]


def pack_problem(problem: object) -> PackedProblem:
    """Derive the verifier's tables from a ``WarpgroupProblem``-shaped object."""
    loop = problem.loop  # type: ignore[attr-defined]
    ops = sorted(loop.ops, key=lambda item: item.id)
    op_ids = tuple(op.id for op in ops)
    if len(set(op_ids)) != len(op_ids):
        raise WarpgroupValidationError("duplicate operation IDs")
    index = {op_id: k for k, op_id in enumerate(op_ids)}

    type_space = {t.id: _space(t.space) for t in problem.types}  # type: ignore[attr-defined]
    space: dict[str, str] = {}
    owner: dict[str, str] = {}
    for item in problem.inputs:  # type: ignore[attr-defined]
        if item.type_id not in type_space:
            raise WarpgroupValidationError(f"input {item.id!r} references undefined type {item.type_id!r}")
        space[item.id] = type_space[item.type_id]
    uses: dict[str, list[str]] = {}
    for op in ops:
        for out in op.outputs:
            if out.id in space:
                raise WarpgroupValidationError(f"duplicate SSA definition {out.id!r}")
            if out.type_id not in type_space:
                raise WarpgroupValidationError(f"output {out.id!r} references undefined type {out.type_id!r}")
            space[out.id] = type_space[out.type_id]
            owner[out.id] = op.id
            uses[out.id] = list(value_references(out.expression))
    carried_from: dict[str, str] = {}
    for arg in loop.iter_args:
        yielded = arg.yield_value.id
        if yielded not in owner:
            raise WarpgroupValidationError(f"iter_arg {arg.id!r} yield must name a loop-body SSA definition")
        if arg.id in space:
            raise WarpgroupValidationError(f"duplicate SSA definition {arg.id!r}")
        space[arg.id] = space[yielded]
        owner[arg.id] = owner[yielded]
        carried_from[arg.id] = owner[yielded]
    inputs = {item.id for item in problem.inputs}  # type: ignore[attr-defined]

    users: dict[str, set[str]] = {}
    relations: set[tuple[int, int, int]] = set()
    for op in ops:
        for out in op.outputs:
            for value in uses[out.id]:
                if value not in space:
                    raise WarpgroupValidationError(f"output {out.id!r} uses undefined SSA value {value!r}")
                users.setdefault(value, set()).add(op.id)
                if value in inputs:
                    continue
                if value in carried_from:
                    relations.add((index[carried_from[value]], index[op.id], 1))
                elif owner[value] != op.id:
                    relations.add((index[owner[value]], index[op.id], 0))
    for op in ops:  # write-after-read reuse of each shared allocation
        for out in op.outputs:
            if space[out.id] != _SPACE_SHARED:
                continue
            for user in users.get(out.id, ()):
                if user != op.id:
                    relations.add((index[user], index[op.id], 1))

    carried: set[tuple[int, int]] = set()
    for arg in loop.iter_args:
        if space[arg.id] != _SPACE_SHARED:
            continue
        defining = owner[arg.id]
        for user in users.get(arg.id, ()):
            if user != defining:
                carried.add((index[user], index[defining]))

    groups: list[list[int]] = []
    for value, value_space in space.items():
        if value_space != _SPACE_REGISTER:
            continue
        members = set(users.get(value, ()))
        if value in owner:
            members.add(owner[value])
        if len(members) > 1:
            groups.append(sorted(index[m] for m in members))
    groups.sort()

    resources = sorted(problem.resources, key=lambda item: item.id)  # type: ignore[attr-defined]
    res_index = {r.id: k for k, r in enumerate(resources)}
    win_off, win_res, win_amt, win_dur = [0], [], [], []
    for op in ops:
        for window in sorted(op.resource_windows, key=lambda w: (w.resource_id, w.amount, w.duration)):
            if window.resource_id not in res_index:
                raise WarpgroupValidationError(f"operation {op.id!r} uses undefined resource {window.resource_id!r}")
            win_res.append(res_index[window.resource_id])
            win_amt.append(window.amount)
            win_dur.append(window.duration)
        win_off.append(len(win_res))

    i32 = lambda values: np.ascontiguousarray(np.array(values, dtype=np.int64).astype(np.int32))  # noqa: E731
    return PackedProblem(
        op_ids=op_ids,
        index=index,
        iterations=int(loop.iterations),
        warp_groups=int(problem.warp_groups),  # type: ignore[attr-defined]
        issue=i32([op.issue_duration for op in ops]),
        latency=i32([op.completion_latency for op in ops]),
        warp_group=i32([-1 if op.warp_group is None else op.warp_group for op in ops]),
        relations=i32(sorted(relations)).reshape(-1, 3),
        carried=i32(sorted(carried)).reshape(-1, 2),
        register_offsets=i32([0] + list(np.cumsum([len(g) for g in groups], dtype=np.int64))),
        register_ops=i32([k for g in groups for k in g]),
        resource_ids=tuple(r.id for r in resources),
        capacity=i32([r.capacity for r in resources]),
        window_offsets=i32(win_off),
        window_resource=i32(win_res),
        window_amount=i32(win_amt),
        window_duration=i32(win_dur),
    )


def _ptr(array: np.ndarray) -> int | None:
    return array.ctypes.data if array.size else None


def problem_desc(packed: PackedProblem, desc_type: type[ctypes.Structure]) -> ctypes.Structure:
    """Fill a ``tfv_problem_desc`` whose pointers stay valid while ``packed`` lives."""
    rel = np.ascontiguousarray(packed.relations.T)  # after, before, distance rows
    car = np.ascontiguousarray(packed.carried.T)
    packed._keep = [rel, car]
    R, C = packed.relations.shape[0], packed.carried.shape[0]
    return desc_type(
        packed.n_ops,
        packed.iterations,
        packed.warp_groups,
        _ptr(packed.issue),
        _ptr(packed.latency),
        _ptr(packed.warp_group),
        R,
        _ptr(rel[0]) if R else None,
        _ptr(rel[1]) if R else None,
        _ptr(rel[2]) if R else None,
        C,
        _ptr(car[0]) if C else None,
        _ptr(car[1]) if C else None,
        len(packed.register_offsets) - 1,
        _ptr(packed.register_offsets),
        _ptr(packed.register_ops),
        len(packed.resource_ids),
        _ptr(packed.capacity),
        _ptr(packed.window_offsets),
        _ptr(packed.window_resource),
        _ptr(packed.window_amount),
        _ptr(packed.window_duration),
    )


__all__ = ["PackedProblem", "pack_problem", "problem_desc"]
