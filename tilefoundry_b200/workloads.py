"""Seeded synthetic candidate batches for benchmarks and tests.

``mla_perturbations`` builds the MLA decode batch: neighbourhood candidates of one
verified witness schedule in compact periodic form. Each candidate is one of

* ``jitter``    — 1 to 3 operations get their prologue and body starts shifted by
                  U[-64, 64] cycles (mostly lane-order or sync failures);
* ``shift``     — every start moves later by a common amount, body starts by up to 64
                  cycles more than prologue starts (stays valid, new makespan);
* ``reassign``  — one operation moves to a random warpgroup at a random position
                  (ownership failures where the operation declares its warp group);
* ``swap``      — two shared-memory producers of one lane exchange positions;
* ``drop_sync`` — one synchronization edge is removed (path failures);
* ``ii``        — the initiation interval changes by U[-40, 40].

Structural variants come from a seeded pool of frames, so a batch holds a few hundred
distinct frames whatever its size. All starts are deltas against the witness.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .batch import FrameSet, PeriodicBatch
from .problem import PackedProblem

MIX = {"jitter": 0.40, "shift": 0.35, "reassign": 0.10, "swap": 0.05, "drop_sync": 0.05, "ii": 0.05}


@dataclass
class Witness:
    """A periodic witness schedule: lanes, sync edges, prologue/offset starts, II."""

    lanes: list[list[str]]
    sync: list[tuple[str, str, int]]
    prologue: np.ndarray  # [N] in problem op order
    offset: np.ndarray
    ii: int


def witness_from_rows(packed: PackedProblem, lanes, sync, rows) -> Witness:
    """Recover the periodic form of a schedule whose body rows are exactly periodic."""
    N, I = packed.n_ops, packed.iterations
    starts = {(r[0], r[1]): r[2] for r in rows}
    ii = starts[(2, packed.op_ids[0])] - starts[(1, packed.op_ids[0])] if I >= 3 else 0
    prologue = np.array([starts[(0, op)] for op in packed.op_ids], dtype=np.int64)
    offset = np.array([starts[(1, op)] - ii for op in packed.op_ids], dtype=np.int64) if I >= 2 else prologue.copy()
    for i in range(1, I):
        for k, op in enumerate(packed.op_ids):
            if starts[(i, op)] != offset[k] + i * ii:
                raise ValueError("witness body rows are not periodic")
    del N
    return Witness([list(l) for l in lanes], [tuple(e) for e in sync], prologue, offset, int(ii))


def _frame_pool(packed: PackedProblem, witness: Witness, shared_producers: set[str], rng: np.random.Generator, size: int):
    pool: dict[str, list[tuple[list, list]]] = {"reassign": [], "swap": [], "drop_sync": []}
    L = len(witness.lanes)
    for _ in range(size):
        lanes = [list(l) for l in witness.lanes]
        op = packed.op_ids[rng.integers(packed.n_ops)]
        for lane in lanes:
            if op in lane:
                lane.remove(op)
        target = int(rng.integers(L))
        lanes[target].insert(int(rng.integers(len(lanes[target]) + 1)), op)
        pool["reassign"].append((lanes, witness.sync))
    for _ in range(size):
        lanes = [list(l) for l in witness.lanes]
        lane = lanes[int(rng.integers(L))]
        slots = [k for k, op in enumerate(lane) if op in shared_producers] or list(range(len(lane)))
        if len(slots) >= 2:
            x, y = rng.choice(slots, size=2, replace=False)
            lane[x], lane[y] = lane[y], lane[x]
        pool["swap"].append((lanes, witness.sync))
    for k in range(min(size, max(1, len(witness.sync)))):
        drop = k % max(1, len(witness.sync))
        pool["drop_sync"].append((witness.lanes, [e for j, e in enumerate(witness.sync) if j != drop]))
    return pool


def shared_producers(problem: object) -> set[str]:
    """Operations with at least one output in shared memory."""
    shared = {t.id for t in problem.types if (t.space.value if hasattr(t.space, "value") else t.space) == "shared"}  # type: ignore[attr-defined]
    return {op.id for op in problem.loop.ops if any(o.type_id in shared for o in op.outputs)}  # type: ignore[attr-defined]


def mla_perturbations(
    packed: PackedProblem,
    witness: Witness,
    n: int,
    *,
    seed: int = 0,
    producers: set[str] | None = None,
    pool_size: int = 64,
    mix: dict[str, float] | None = None,
) -> tuple[FrameSet, PeriodicBatch, np.ndarray]:
    """``n`` seeded neighbourhood candidates of ``witness``; returns frames, batch, kind ids."""
    mix = mix or MIX
    rng = np.random.default_rng(seed)
    N = packed.n_ops
    frames = FrameSet(packed)
    base_frame = frames.add(witness.lanes, witness.sync)
    pool = _frame_pool(packed, witness, producers or set(), rng, pool_size)
    pool_ids = {kind: np.array([frames.add(l, s) for l, s in entries], dtype=np.int32) for kind, entries in pool.items()}

    kinds = list(mix)
    probs = np.array([mix[k] for k in kinds], dtype=np.float64)
    kind = rng.choice(len(kinds), size=n, p=probs / probs.sum()).astype(np.int8)
    dp = np.zeros((N, n), dtype=np.int16)
    dq = np.zeros((N, n), dtype=np.int16)
    ii = np.full(n, witness.ii, dtype=np.int32)
    frame = np.full(n, base_frame, dtype=np.int32)

    sel = np.flatnonzero(kind == kinds.index("jitter"))
    if sel.size:
        count = rng.integers(1, 4, size=sel.size)
        for j in range(3):
            rows = sel[count > j]
            ops = rng.integers(0, N, size=rows.size)
            dp[ops, rows] += rng.integers(-64, 65, size=rows.size).astype(np.int16)
            dq[ops, rows] += rng.integers(-64, 65, size=rows.size).astype(np.int16)
    sel = np.flatnonzero(kind == kinds.index("shift"))
    if sel.size:
        s1 = rng.integers(0, 401, size=sel.size).astype(np.int16)
        s2 = rng.integers(0, 65, size=sel.size).astype(np.int16)
        dp[:, sel] = s1[None, :]
        dq[:, sel] = (s1 + s2)[None, :]
    for name in ("reassign", "swap", "drop_sync"):
        sel = np.flatnonzero(kind == kinds.index(name))
        if sel.size and pool_ids[name].size:
            frame[sel] = pool_ids[name][rng.integers(0, pool_ids[name].size, size=sel.size)]
    sel = np.flatnonzero(kind == kinds.index("ii"))
    if sel.size:
        ii[sel] += rng.integers(-40, 41, size=sel.size).astype(np.int32)

    batch = PeriodicBatch(
        base_prologue=witness.prologue.astype(np.int32),
        base_offset=witness.offset.astype(np.int32),
        prologue_delta=dp,
        offset_delta=dq,
        ii=ii,
        frame=frame,
    )
    return frames, batch, kind


def absolute_starts(batch: PeriodicBatch) -> tuple[np.ndarray, np.ndarray]:
    """[n, N] int64 prologue and offset starts of a periodic batch."""
    prologue = batch.base_prologue.astype(np.int64)[None, :] + batch.prologue_delta.T.astype(np.int64)
    offset = batch.base_offset.astype(np.int64)[None, :] + batch.offset_delta.T.astype(np.int64)
    return prologue, offset


__all__ = [
    "BODIES", "MIX", "Witness", "absolute_starts", "body_batch", "mla_perturbations", "peak_demands", "pipelined_batch",
    "pipelined_starts", "shared_producers", "witness_from_rows", "with_capacities",
]


# ---------------------------------------------------------------------------------------
# Random layered DAG problems and list-scheduled witnesses
# ---------------------------------------------------------------------------------------


def random_dag_problem(
    n_ops: int = 256,
    *,
    layers: int = 16,
    lanes: int = 8,
    n_resources: int = 6,
    iterations: int = 32,
    seed: int = 0,
    latency: tuple[int, int] = (20, 2000),
    fan_in: tuple[int, int] = (1, 4),
    capacity: tuple[int, int] = (4, 64),
    demand: tuple[int, int] = (1, 8),
    windows_per_op: tuple[int, int] = (0, 2),
    declared: float = 1.0,
    carried: float = 0.05,
    pareto_alpha: float | None = None,
):
    """A seeded layered DAG problem (mirror records).

    Operation k sits in layer ``k * layers // n_ops`` and reads 1-4 values of earlier
    layers (layer 0 reads the external input). With probability ``carried`` an
    operation also reads a loop-carried value yielded by an operation of a later layer
    (a distance-1 dependency). A value is a register value when its producer and all
    users declare the same warp group, otherwise it lives in shared memory. Resource
    demands are uniform, or Pareto(``pareto_alpha``) capped at the capacity.
    """
    from .model import (
        LoopIterArg,
        OperationOutput,
        ProblemLoop,
        ProblemOperation,
        ProgramInput,
        ResourceCapacity,
        ResourceWindow,
        TensorType,
        ValueRef,
        ValueUses,
        WarpgroupProblem,
    )

    rng = np.random.default_rng(seed)
    layer = [k * layers // n_ops for k in range(n_ops)]
    wg = [int(rng.integers(lanes)) if rng.random() < declared else None for _ in range(n_ops)]
    lat = [int(rng.integers(latency[0], latency[1] + 1)) for _ in range(n_ops)]
    issue = [int(rng.integers(1, max(1, v // 4) + 1)) for v in lat]
    reads: list[list[str]] = []
    for k in range(n_ops):
        earlier = [j for j in range(n_ops) if layer[j] < layer[k]]
        if not earlier:
            reads.append(["%in"])
            continue
        count = int(rng.integers(fan_in[0], fan_in[1] + 1))
        picks = rng.choice(len(earlier), size=min(count, len(earlier)), replace=False)
        reads.append([f"%v{earlier[int(j)]}" for j in sorted(picks)])
    iter_args: list[tuple[str, int]] = []
    for k in range(n_ops):
        later = [j for j in range(n_ops) if layer[j] > layer[k]]
        if later and rng.random() < carried:
            y = later[int(rng.integers(len(later)))]
            name = f"%c{len(iter_args)}"
            iter_args.append((name, y))
            reads[k].append(name)
    users: dict[str, set[int]] = {}
    for k, values in enumerate(reads):
        for v in values:
            users.setdefault(v, set()).add(k)
    space: dict[str, str] = {}
    for k in range(n_ops):
        group = {k} | users.get(f"%v{k}", set())
        for name, y in iter_args:
            if y == k:
                group |= users.get(name, set())
        owners = {wg[j] for j in group}
        space[f"%v{k}"] = "register" if len(owners) == 1 and None not in owners else "shared"
    caps = [int(rng.integers(capacity[0], capacity[1] + 1)) for _ in range(n_resources)]
    resources = tuple(ResourceCapacity(f"res{q}", caps[q]) for q in range(n_resources))
    ops = []
    for k in range(n_ops):
        windows = []
        if n_resources:
            for _ in range(int(rng.integers(windows_per_op[0], windows_per_op[1] + 1))):
                q = int(rng.integers(n_resources))
                if pareto_alpha is None:
                    amount = int(rng.integers(demand[0], demand[1] + 1))
                else:
                    amount = int(np.ceil(demand[0] * (1.0 + rng.pareto(pareto_alpha))))
                held = sum(w.amount for w in windows if w.resource_id == f"res{q}")
                amount = max(1, min(amount, caps[q] - held))
                if held >= caps[q]:
                    continue
                windows.append(ResourceWindow(f"res{q}", amount, int(rng.integers(1, lat[k] + 1))))
        kind = "reg" if space[f"%v{k}"] == "register" else "smem"
        ops.append(
            ProblemOperation(
                f"op{k:04d}",
                (OperationOutput(f"%v{k}", kind, ValueUses(tuple(reads[k]))),),
                wg[k],
                issue[k],
                lat[k],
                tuple(windows),
            )
        )
    types = (TensorType("gmem", "global"), TensorType("reg", "register"), TensorType("smem", "shared"))
    return WarpgroupProblem(
        "cycle",
        lanes,
        resources,
        types,
        (ProgramInput("%in", "gmem"),),
        ProblemLoop("%i", iterations, tuple(LoopIterArg(name, ValueRef(f"%v{y}")) for name, y in iter_args), tuple(ops)),
    )


def list_schedule_witness(packed: PackedProblem, *, seed: int = 0, lane_of: list[int] | None = None) -> Witness:
    """A valid periodic witness by list scheduling one iteration.

    Lanes follow the declared warp groups (undeclared operations get a seeded lane);
    each lane runs its operations in a topological order of the same-iteration
    constraints (distance-0 relations and carried-lifetime pairs). Operations start as early as
    their lane predecessor's issue end, their distance-0 relations' completions, the
    carried-lifetime users' completions and the resource capacities allow. Body
    iterations repeat the prologue one span later (offset = prologue, II = span), so
    iterations never overlap and every cross-iteration constraint holds. The sync set
    is every required relation with a finite instance.
    """
    rng = np.random.default_rng(seed)
    N, L, I = packed.n_ops, packed.warp_groups, packed.iterations
    if lane_of is None:
        lane_of = [int(w) if w >= 0 else int(rng.integers(L)) for w in packed.warp_group]
    preds: list[list[int]] = [[] for _ in range(N)]
    for a, b, d in packed.relations:
        if d == 0:
            preds[int(b)].append(int(a))
    for u, df in packed.carried:
        preds[int(df)].append(int(u))
    windows = [
        [(int(packed.window_resource[w]), int(packed.window_amount[w]), int(packed.window_duration[w]))
         for w in range(packed.window_offsets[k], packed.window_offsets[k + 1])]
        for k in range(N)
    ]
    placed: dict[int, list[tuple[int, int, int]]] = {q: [] for q in range(len(packed.resource_ids))}
    start = np.zeros(N, dtype=np.int64)
    lane_tail: dict[int, int] = {}

    def fits(t: int, k: int) -> bool:
        for q in {w[0] for w in windows[k]}:
            own = [(amount, dur) for r, amount, dur in windows[k] if r == q]
            reach = max(dur for _, dur in own)
            points = [t] + [s for s, e, _ in placed[q] if t <= s < t + reach]
            for p in points:
                used = sum(a for s, e, a in placed[q] if s <= p < e)
                used += sum(amount for amount, dur in own if p < t + dur)
                if used > int(packed.capacity[q]):
                    return False
        return True

    # Kahn's algorithm over the same-iteration constraints, smallest index first.
    import heapq

    succs: list[list[int]] = [[] for _ in range(N)]
    indeg = [0] * N
    for k in range(N):
        for a in preds[k]:
            succs[a].append(k)
            indeg[k] += 1
    ready = [k for k in range(N) if indeg[k] == 0]
    heapq.heapify(ready)
    topo: list[int] = []
    while ready:
        k = heapq.heappop(ready)
        topo.append(k)
        for b in succs[k]:
            indeg[b] -= 1
            if indeg[b] == 0:
                heapq.heappush(ready, b)
    if len(topo) != N:
        raise ValueError("same-iteration constraints are cyclic: no single-iteration witness exists")
    for k in topo:
        for q in {w[0] for w in windows[k]}:
            if sum(amount for r, amount, _ in windows[k] if r == q) > int(packed.capacity[q]):
                raise ValueError(f"operation {packed.op_ids[k]!r} alone exceeds resource {packed.resource_ids[q]!r}")
        t = 0
        if lane_of[k] in lane_tail:
            prev = lane_tail[lane_of[k]]
            t = max(t, int(start[prev] + packed.issue[prev]))
        for a in preds[k]:
            t = max(t, int(start[a] + packed.latency[a]))
        while not fits(t, k):
            t += 1 + int(rng.integers(0, 8))
        start[k] = t
        for q, amount, dur in windows[k]:
            placed[q].append((t, t + dur, amount))
        lane_tail[lane_of[k]] = k
    span = int((start + packed.latency).max())
    lanes = [[packed.op_ids[k] for k in topo if lane_of[k] == l] for l in range(L)]
    sync = [(packed.op_ids[a], packed.op_ids[b], int(d)) for a, b, d in packed.relations if d < I]
    return Witness(lanes, sync, start.copy(), start.copy(), max(span, 1))


def neighbourhood(
    packed: PackedProblem,
    witness: Witness,
    n: int,
    *,
    seed: int = 0,
    jitter: int = 64,
    tighten: float = 0.5,
    pool_size: int = 32,
) -> tuple[FrameSet, PeriodicBatch]:
    """Seeded periodic neighbours of a witness: jittered starts, tightened II, new frames.

    A quarter of the candidates keep the witness times shifted later (valid), a
    quarter jitter a few operations, a quarter tighten the II by up to ``tighten`` of
    the span (overlapping iterations: lane wrap, distance-1 and resource checks), and
    the rest use a structural variant (moved operation, swapped lane neighbours or a
    dropped sync edge) with jittered times.
    """
    rng = np.random.default_rng(seed)
    N = packed.n_ops
    frames = FrameSet(packed)
    base = frames.add(witness.lanes, witness.sync)
    variants = []
    for _ in range(pool_size):
        lanes = [list(l) for l in witness.lanes]
        sync = list(witness.sync)
        roll = rng.random()
        nonempty = [l for l in lanes if len(l) >= 2] or lanes
        if roll < 0.34:
            op = packed.op_ids[int(rng.integers(N))]
            for lane in lanes:
                if op in lane:
                    lane.remove(op)
            target = lanes[int(rng.integers(len(lanes)))]
            target.insert(int(rng.integers(len(target) + 1)), op)
        elif roll < 0.67:
            lane = nonempty[int(rng.integers(len(nonempty)))]
            if len(lane) >= 2:
                x = int(rng.integers(len(lane) - 1))
                lane[x], lane[x + 1] = lane[x + 1], lane[x]
        elif sync:
            sync.pop(int(rng.integers(len(sync))))
        variants.append(frames.add(lanes, sync))
    variants = np.array(variants, dtype=np.int32)
    kind = rng.integers(0, 4, size=n)
    dp = np.zeros((N, n), dtype=np.int64)
    dq = np.zeros((N, n), dtype=np.int64)
    ii = np.full(n, witness.ii, dtype=np.int64)
    frame = np.full(n, base, dtype=np.int32)
    shift = rng.integers(0, jitter + 1, size=n)
    sel = kind == 0
    dp[:, sel] = shift[sel]
    dq[:, sel] = shift[sel] + rng.integers(0, jitter + 1, size=int(sel.sum()))
    for sel in (kind == 1, kind == 3):
        rows = np.flatnonzero(sel)
        for _ in range(3):
            ops = rng.integers(0, N, size=rows.size)
            dp[ops, rows] += rng.integers(-jitter, jitter + 1, size=rows.size)
            dq[ops, rows] += rng.integers(-jitter, jitter + 1, size=rows.size)
    sel = kind == 2
    ii[sel] -= (rng.random(int(sel.sum())) * tighten * witness.ii).astype(np.int64)
    sel = np.flatnonzero(kind == 3)
    if variants.size:
        frame[sel] = variants[rng.integers(0, variants.size, size=sel.size)]
    batch = PeriodicBatch(
        base_prologue=witness.prologue.astype(np.int32),
        base_offset=witness.offset.astype(np.int32),
        prologue_delta=np.ascontiguousarray(dp.astype(np.int16)),
        offset_delta=np.ascontiguousarray(dq.astype(np.int16)),
        ii=ii.astype(np.int32),
        frame=frame,
    )
    return frames, batch


# ---------------------------------------------------------------------------------------
# Kernel-body problems: GEMM mainloop and FlashAttention forward
# ---------------------------------------------------------------------------------------


def _body_problem(ops_spec, lanes: int, iterations: int, capacities: dict, iter_args=(), inputs=("%gmem",)):
    """Closed problem from ``(id, warp_group, issue, latency, [(resource, amount, duration)], out, space, uses)``."""
    from .model import (
        LoopIterArg,
        OperationOutput,
        ProblemLoop,
        ProblemOperation,
        ProgramInput,
        ResourceCapacity,
        ResourceWindow,
        TensorType,
        ValueRef,
        ValueUses,
        WarpgroupProblem,
    )

    kinds = {"register": "reg", "shared": "smem"}
    ops = tuple(
        ProblemOperation(
            op_id,
            (OperationOutput(out, kinds[space], ValueUses(tuple(uses))),),
            wg,
            issue,
            latency,
            tuple(ResourceWindow(r, a, d) for r, a, d in windows),
        )
        for op_id, wg, issue, latency, windows, out, space, uses in ops_spec
    )
    return WarpgroupProblem(
        "cycle",
        lanes,
        tuple(ResourceCapacity(r, c) for r, c in capacities.items()),
        (TensorType("gmem", "global"), TensorType("reg", "register"), TensorType("smem", "shared")),
        tuple(ProgramInput(i, "gmem") for i in inputs),
        ProblemLoop("%iter", iterations, tuple(LoopIterArg(a, ValueRef(y)) for a, y in iter_args), ops),
    )


def gemm_mainloop_problem(iterations: int = 8):
    """GEMM mainloop body: TMA loads of A (128x64 bf16, 16 KB) and B (256x64 bf16, 32 KB)
    by the producer warpgroup, a 128x256x64 tcgen05 MMA (latency 512) and a barrier
    arrive by the consumer, and an epilogue store of the 128x256 fp32 accumulator.
    Resources: shared memory in KB (227), TMEM columns (512), mbarriers (8) and the slots
    of the 4-stage A/B ring (8: a stage holds one A and one B tile). As in the reference's
    model each loaded tile is one shared allocation, reused by the next iteration's load
    once this iteration's MMA has completed; the accumulator belongs to the MMA warpgroup (a
    register value carried from one iteration's MMA to the next). The MMA's recurrence bounds
    the work in flight, so these capacities are never exceeded by a candidate that keeps its
    lane, sync and relation inequalities (the calibrated variant of body_batch tightens
    them)."""
    spec = [
        ("load_a", 0, 24, 700, [("smem_kb", 16, 700), ("tma_slots", 1, 700)], "%a", "shared", ["%gmem"]),
        ("load_b", 0, 24, 900, [("smem_kb", 32, 900), ("tma_slots", 1, 900)], "%b", "shared", ["%gmem"]),
        ("mma", 1, 64, 512, [("tmem_cols", 256, 512), ("mbarrier", 1, 512)], "%acc", "register",
         ["%a", "%b", "%acc_prev"]),
        ("arrive", 1, 4, 4, [("mbarrier", 1, 4)], "%bar", "register", ["%acc"]),
        ("store", 1, 160, 420, [("smem_kb", 96, 420)], "%out", "register", ["%acc", "%bar"]),
    ]
    caps = {"smem_kb": 227, "tmem_cols": 512, "mbarrier": 8, "tma_slots": 8}
    return _body_problem(spec, 2, iterations, caps, iter_args=[("%acc_prev", "%acc")])


def flash_attention_problem(iterations: int = 16):
    """FlashAttention-forward body (Q 128x128, K/V 128x128 bf16 tiles): loads of K and V
    (load warpgroup), S = QK^T and P.V MMAs (MMA warpgroup), rowmax, exp2, rowsum and the O
    rescale (softmax warpgroup). Shared memory 227 KB, TMEM 512 columns. As for the GEMM
    body, the recurrences bound the work in flight below the nominal capacities."""
    spec = [
        ("load_k", 0, 24, 800, [("smem_kb", 32, 800)], "%k", "shared", ["%gmem"]),
        ("load_v", 0, 24, 800, [("smem_kb", 32, 800)], "%v", "shared", ["%gmem"]),
        ("qk", 1, 48, 384, [("tmem_cols", 128, 384)], "%s", "shared", ["%gmem", "%k"]),
        ("rowmax", 2, 90, 110, [], "%m", "register", ["%s", "%m_prev"]),
        ("exp2", 2, 220, 240, [("smem_kb", 32, 240)], "%p", "shared", ["%s", "%m"]),
        ("rowsum", 2, 80, 96, [], "%l", "register", ["%p", "%l_prev"]),
        ("rescale", 2, 140, 160, [("tmem_cols", 128, 160)], "%o_scaled", "shared", ["%o_prev", "%m", "%m_prev"]),
        ("pv", 1, 48, 384, [("tmem_cols", 128, 384)], "%o", "shared", ["%p", "%v", "%o_scaled"]),
    ]
    caps = {"smem_kb": 227, "tmem_cols": 512}
    return _body_problem(
        spec, 3, iterations, caps, iter_args=[("%m_prev", "%m"), ("%l_prev", "%l"), ("%o_prev", "%o")]
    )


def dag_problem(seed: int = 0):
    """Random layered DAG: 256 ops in 16 layers, fan-in 1-4, latencies U[20, 2000],
    8 warpgroups, 6 resources with capacities U[4, 64] and demands 1-8, 32 iterations."""
    return random_dag_problem(256, layers=16, lanes=8, n_resources=6, iterations=32, seed=seed)


def stress_problem(seed: int = 0):
    """Stress body: a 1024-op random DAG (same generator), 12 warpgroups, 64 iterations,
    heavy-tailed demands (Pareto alpha = 1.5, capped at the capacity)."""
    return random_dag_problem(
        1024, layers=32, lanes=12, n_resources=6, iterations=64, seed=seed, pareto_alpha=1.5, demand=(1, 8)
    )


def ii_lower_bound(packed: PackedProblem) -> int:
    """The solver's II lower bound: the longest issue duration, and per resource the
    held amount-cycles of one iteration over its capacity, rounded up
    (solve.py:186-204, 261-264)."""
    bound = int(packed.issue.max()) if packed.n_ops else 1
    held: dict[int, int] = {}
    for w in range(len(packed.window_resource)):
        q = int(packed.window_resource[w])
        held[q] = held.get(q, 0) + int(packed.window_duration[w]) * int(packed.window_amount[w])
    for q, total in held.items():
        bound = max(bound, -(-total // int(packed.capacity[q])))
    return max(bound, 1)


def ii_sweep(ii_lb: int, n_ii: int = 16) -> np.ndarray:
    """``n_ii`` initiation intervals spread evenly over [ii_lb, 2 * ii_lb]."""
    if n_ii == 1:
        return np.array([ii_lb], dtype=np.int64)
    return ii_lb + (np.arange(n_ii, dtype=np.int64) * ii_lb) // (n_ii - 1)


# ---------------------------------------------------------------------------------------
# Software-pipelined candidates: overlapping iterations decided by the resource capacities
# ---------------------------------------------------------------------------------------


def _constraint_lists(packed: PackedProblem, lanes: list[list[str]]):
    """Difference constraints of a periodic schedule with fixed lanes (verify.py:278-318).

    Returns the same-iteration topological order and, per operation b, its same-iteration
    predecessors ``(a, weight)`` (lane predecessor with a's issue duration, distance-0
    relations with a's latency), its body-only predecessors (carried shared lifetimes, which
    hold in iterations 1..I-1) and its next-iteration predecessors (distance-1 relations
    and the lane wrap from a lane's last operation to its first).
    """
    N = packed.n_ops
    same: list[list[tuple[int, int]]] = [[] for _ in range(N)]
    body: list[list[tuple[int, int]]] = [[] for _ in range(N)]
    nxt: list[list[tuple[int, int]]] = [[] for _ in range(N)]
    for lane in lanes:
        ks = [packed.index[op] for op in lane]
        for a, b in zip(ks, ks[1:]):
            same[b].append((a, int(packed.issue[a])))
        if ks:
            nxt[ks[0]].append((ks[-1], int(packed.issue[ks[-1]])))
    for a, b, d in packed.relations:
        (same if d == 0 else nxt)[int(b)].append((int(a), int(packed.latency[a])))
    for u, df in packed.carried:
        body[int(df)].append((int(u), int(packed.latency[u])))
    indeg = [0] * N
    succs: list[list[int]] = [[] for _ in range(N)]
    for b in range(N):
        for a, _ in same[b] + body[b]:
            succs[a].append(b)
            indeg[b] += 1
    order = [k for k in range(N) if indeg[k] == 0]
    for k in order:
        for b in succs[k]:
            indeg[b] -= 1
            if indeg[b] == 0:
                order.append(b)
    if len(order) != N:
        raise ValueError("the lanes and same-iteration relations are cyclic")
    return order, same, body, nxt


def pipelined_starts(packed: PackedProblem, lanes, ii: np.ndarray, delay_p: np.ndarray, delay_o: np.ndarray,
                     rounds: int | None = None, floor_p: np.ndarray | None = None, floor_o: np.ndarray | None = None):
    """Earliest prologue and body-offset starts of periodic schedules at the given IIs.

    ``ii`` is [n]; ``delay_p``/``delay_o`` [n, N] non-negative extra delays; ``floor_p`` /
    ``floor_o`` ([n, N] or [N]) optional earliest starts of each operation. The prologue
    (iteration 0, solve.py:215-217) is scheduled as soon as its same-iteration constraints
    allow; the body offsets (iterations >= 1 start at offset + i * II, solve.py:218-221) are
    the least solution of every constraint at that II, including those from iteration 0 to
    iteration 1, by Bellman-Ford rounds. Returns ``(prologue, offset, feasible)``: a
    candidate is feasible when the rounds converged (no positive cycle at its II); feasible
    candidates satisfy every lane, sync, relation and carried-lifetime inequality with the
    full relation set as sync, so the resource capacities decide their verdict.
    """
    order, same, body, nxt = _constraint_lists(packed, lanes)
    n, N = delay_p.shape
    ii = np.asarray(ii, dtype=np.int64)
    fp = np.broadcast_to(np.zeros(N, dtype=np.int64) if floor_p is None else np.asarray(floor_p, np.int64), (n, N))
    fo = np.broadcast_to(np.zeros(N, dtype=np.int64) if floor_o is None else np.asarray(floor_o, np.int64), (n, N))
    p = np.zeros((n, N), dtype=np.int64)
    for b in order:
        t = fp[:, b].copy()
        for a, w in same[b]:
            t = np.maximum(t, p[:, a] + w)
        p[:, b] = t + delay_p[:, b]
    o = fo + delay_o.astype(np.int64)  # body rows start no earlier than cycle ii
    live = np.ones(n, dtype=bool)
    limit = rounds if rounds is not None else N + 2
    for _ in range(limit):
        before = o.copy()
        for b in order:
            t = o[:, b]
            for a, w in same[b]:
                t = np.maximum(t, o[:, a] + w)
            for a, w in body[b]:
                t = np.maximum(t, o[:, a] + w)
            for a, w in nxt[b]:
                t = np.maximum(t, np.maximum(p[:, a], o[:, a]) + w - ii)
            o[:, b] = t
        changed = (o != before).any(axis=1)
        if not changed.any():
            break
    else:
        changed = (o != before).any(axis=1)
        live &= ~changed
    return p, o, live


def pipelined_batch(
    packed: PackedProblem,
    witness: Witness,
    n: int,
    *,
    seed: int = 0,
    ii_range: tuple[int, int] | None = None,
    delay: float = 0.1,
    delay_scale: int = 200,
    start_range: int | None = None,
    corrupt: float = 0.5,
    jitter: int = 64,
    pool: int = 2048,
    pool_size: int = 32,
) -> tuple[FrameSet, PeriodicBatch, np.ndarray]:
    """``n`` seeded software-pipelined candidates around the witness's lanes.

    A pool of ``pool`` templates is drawn first, each with sparse random delays
    (probability ``delay`` per operation, exponential with mean ``delay_scale`` cycles) and
    the earliest starts that satisfy every lane, sync, relation and carried constraint at
    its II (:func:`pipelined_starts`). Half the templates are pipelined: an II uniform in
    ``ii_range`` (default [II_lb, witness II]) and every start at most 30% of the witness II
    before the witness's, so iterations overlap whenever the II is below the span and every
    template's starts stay within one int16 delta range. The other half keep every start at or after the
    witness's (its resource-feasible single iteration), without delays, at an II uniform in
    [0.9, 1.3] times the witness II. Either way the resource capacities decide between
    verdicts 0 and 20.
    Every candidate takes a template
    and moves all its starts later by a common shift (up to ``start_range`` minus the
    template's largest start, so starts stay in [0, ``start_range``] when given). A fraction
    ``corrupt`` of the candidates is then broken in one of four ways: 1-3 operations
    jittered by U[-jitter, jitter] (lane order, sync and relation timing), the II cut by up
    to a third (wrap edges and distance-1 relations, more overlap), a structural variant
    (an operation moved to another lane, two lane neighbours swapped or a sync edge dropped)
    or one resource-holding operation moved onto another's start, at most 12000 cycles away
    (capacity). Returns the
    frames, the batch and each candidate's kind (0 = uncorrupted, 1-4 as listed).
    """
    rng = np.random.default_rng(seed)
    N = packed.n_ops
    lo, hi = ii_range if ii_range is not None else (ii_lower_bound(packed), max(ii_lower_bound(packed), witness.ii))
    m = max(2, min(pool, n))
    floored = np.arange(m) % 2 == 1
    t_ii = np.where(floored, rng.integers(int(0.9 * witness.ii), int(1.3 * witness.ii) + 2, size=m),
                    rng.integers(lo, hi + 1, size=m))
    sparse = (rng.random((2, m, N)) < delay) & ~floored[None, :, None]
    dp = np.where(sparse[0], rng.exponential(delay_scale, size=(m, N)), 0).astype(np.int64)
    dq = np.where(sparse[1], rng.exponential(delay_scale, size=(m, N)), 0).astype(np.int64)
    # pipelined templates may move each operation up to 30% of the witness II earlier than the
    # witness (its lanes compress, so IIs below the span become feasible); floored ones none
    wp = witness.prologue.astype(np.int64)[None, :]
    floor = np.where(floored[:, None], wp, np.maximum(0, wp - int(0.3 * witness.ii)))
    tp, to, ok = pipelined_starts(packed, witness.lanes, t_ii, dp, dq, floor_p=floor, floor_o=floor)
    keep = np.flatnonzero(ok)
    if keep.size == 0:
        raise ValueError("no template converged: the II range is below every recurrence bound")
    tp, to, t_ii = tp[keep], to[keep], t_ii[keep]
    pick = rng.integers(0, keep.size, size=n)
    top = np.maximum(tp.max(axis=1), to.max(axis=1) + t_ii)[pick]
    room = np.maximum(0, (start_range - top) if start_range is not None else np.full(n, 64))
    shift = (rng.random(n) * (room + 1)).astype(np.int64)
    ii = t_ii[pick].copy()

    frames = FrameSet(packed)
    base = frames.add(witness.lanes, witness.sync)
    frame = np.full(n, base, dtype=np.int32)
    kind = np.where(rng.random(n) < corrupt, rng.integers(1, 5, size=n), 0).astype(np.int8)
    # kind 1: up to three (operation, prologue shift, offset shift) triples per candidate
    jit = np.flatnonzero(kind == 1)
    jit_use = rng.random((3, jit.size)) < 0.7
    jit_op = rng.integers(0, N, size=(3, jit.size))
    jit_dp = rng.integers(-jitter, jitter + 1, size=(3, jit.size))
    jit_dq = rng.integers(-jitter, jitter + 1, size=(3, jit.size))
    sel = np.flatnonzero(kind == 2)
    ii[sel] -= (rng.random(sel.size) * ii[sel] / 3).astype(np.int64)
    sel = np.flatnonzero(kind == 3)
    if sel.size:
        variants = []
        for _ in range(pool_size):
            lanes = [list(l) for l in witness.lanes]
            sync = list(witness.sync)
            roll = rng.random()
            if roll < 0.34:
                op = packed.op_ids[int(rng.integers(N))]
                for lane in lanes:
                    if op in lane:
                        lane.remove(op)
                target = lanes[int(rng.integers(len(lanes)))]
                target.insert(int(rng.integers(len(target) + 1)), op)
            elif roll < 0.67:
                nonempty = [l for l in lanes if len(l) >= 2] or lanes
                lane = nonempty[int(rng.integers(len(nonempty)))]
                if len(lane) >= 2:
                    x = int(rng.integers(len(lane) - 1))
                    lane[x], lane[x + 1] = lane[x + 1], lane[x]
            elif sync:
                sync.pop(int(rng.integers(len(sync))))
            variants.append(frames.add(lanes, sync))
        frame[sel] = np.array(variants, dtype=np.int32)[rng.integers(0, len(variants), size=sel.size)]
    # kind 4: one resource-holding operation moved onto another's starts
    sq = np.flatnonzero(kind == 4)
    holders = np.flatnonzero(np.diff(packed.window_offsets) > 0)
    if holders.size < 2:
        sq = sq[:0]
    sq_a = holders[rng.integers(0, max(1, holders.size), size=sq.size)] if sq.size else sq
    sq_b = holders[rng.integers(0, max(1, holders.size), size=sq.size)] if sq.size else sq

    # Materialise int16 deltas chunk by chunk against per-operation bases at the middle of the
    # templates' range (shifts, jitter and squeezes stay well inside the int16 range).
    base_p = (tp.min(axis=0) + tp.max(axis=0) + 2 * (int(shift.max()) // 2 if n else 0)) // 2
    base_o = (to.min(axis=0) + to.max(axis=0) + 2 * (int(shift.max()) // 2 if n else 0)) // 2
    dp_all = np.empty((N, n), dtype=np.int16)
    dq_all = np.empty((N, n), dtype=np.int16)
    chunk = max(1, (1 << 22) // max(1, N))
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        prologue = tp[pick[c0:c1]] + shift[c0:c1, None]
        offset = to[pick[c0:c1]] + shift[c0:c1, None]
        lo_j, hi_j = np.searchsorted(jit, [c0, c1])
        for r in range(3):
            rows = jit[lo_j:hi_j][jit_use[r, lo_j:hi_j]]
            ops = jit_op[r, lo_j:hi_j][jit_use[r, lo_j:hi_j]]
            prologue[rows - c0, ops] += jit_dp[r, lo_j:hi_j][jit_use[r, lo_j:hi_j]]
            offset[rows - c0, ops] += jit_dq[r, lo_j:hi_j][jit_use[r, lo_j:hi_j]]
        lo_s, hi_s = np.searchsorted(sq, [c0, c1])
        rows = sq[lo_s:hi_s] - c0
        for arr in (offset, prologue):  # at most 12000 cycles, to stay inside the delta range
            a_now = arr[rows, sq_a[lo_s:hi_s]]
            arr[rows, sq_a[lo_s:hi_s]] = np.clip(arr[rows, sq_b[lo_s:hi_s]], a_now - 12000, a_now + 12000)
        d1 = prologue - base_p[None, :]
        d2 = offset - base_o[None, :]
        if min(d1.min(), d2.min()) < -32768 or max(d1.max(), d2.max()) > 32767:
            raise ValueError("candidate starts leave the int16 range around their bases")
        dp_all[:, c0:c1] = d1.T
        dq_all[:, c0:c1] = d2.T
    batch = PeriodicBatch(base_p.astype(np.int32), base_o.astype(np.int32), dp_all, dq_all, ii.astype(np.int32), frame)
    return frames, batch, kind


def peak_demands(packed: PackedProblem, prologue: np.ndarray, offset: np.ndarray, ii: np.ndarray) -> np.ndarray:
    """[n, Q] largest demand of every resource over each periodic candidate's timeline.

    The netted sweep of verify.py:183-200 on every candidate at once (numpy; meant for
    bodies with a few hundred windows at most): +amount at each window copy's start,
    -amount at its end, summed in time order with ends before starts at equal times.
    """
    n = prologue.shape[0]
    I, Q = packed.iterations, len(packed.resource_ids)
    out = np.zeros((n, Q), dtype=np.int64)
    i = np.arange(I, dtype=np.int64)
    starts = offset[:, None, :] + i[None, :, None] * np.asarray(ii, dtype=np.int64)[:, None, None]
    starts[:, 0, :] = prologue
    ops = np.repeat(np.arange(packed.n_ops), np.diff(packed.window_offsets))
    for q in range(Q):
        w = np.flatnonzero(packed.window_resource == q)
        if w.size == 0:
            continue
        s = starts[:, :, ops[w]].reshape(n, -1)
        e = s + np.tile(packed.window_duration[w].astype(np.int64), I)
        a = np.tile(packed.window_amount[w].astype(np.int64), I)
        t = np.concatenate([s, e], axis=1)
        d = np.concatenate([np.broadcast_to(a, s.shape), -np.broadcast_to(a, s.shape)], axis=1)
        order = np.argsort(t * 2 + (d > 0), axis=1, kind="stable")  # ends before starts at equal times
        out[:, q] = np.cumsum(np.take_along_axis(d, order, axis=1), axis=1).max(axis=1)
    return out


def with_capacities(problem: object, capacities: dict[str, int]) -> object:
    """``problem`` (mirror records) with the named resources' capacities replaced."""
    import dataclasses

    resources = tuple(dataclasses.replace(r, capacity=int(capacities.get(r.id, r.capacity)))
                      for r in problem.resources)  # type: ignore[attr-defined]
    return dataclasses.replace(problem, resources=resources)


BODIES = {
    "gemm": gemm_mainloop_problem,
    "fa": flash_attention_problem,
    "dag": dag_problem,
    "stress": stress_problem,
}


def body_batch(name: str, n: int, *, seed: int = 0, calibrated: bool = False, pool: int = 2048):
    """A seeded batch of ``n`` candidates for one of the kernel-body problems.

    ``name`` is ``gemm`` (starts in [0, 8000]), ``fa``, ``dag`` or ``stress``; candidates
    come from :func:`pipelined_batch` with half of them corrupted. With ``calibrated`` the
    problem's capacities are set to the median of the uncorrupted candidates' peak demands
    (:func:`peak_demands`), so that each resource whose peak varies is exceeded by part of
    the batch:
    with the nominal capacities of the GEMM and FlashAttention bodies no candidate that
    keeps the lane, sync and relation inequalities can exceed them (their recurrences bound
    the work in flight). Returns ``(problem, packed, witness, frames, batch, kind)``.
    """
    from .problem import pack_problem

    problem = BODIES[name]()
    packed = pack_problem(problem)
    witness = list_schedule_witness(packed, seed=1)
    frames, batch, kind = pipelined_batch(packed, witness, n, seed=seed, pool=min(pool, max(2, n)),
                                          start_range=8000 if name == "gemm" else None)
    if calibrated:
        p, o = absolute_starts(batch)
        clean = np.flatnonzero(kind == 0)[:4096]
        peaks = peak_demands(packed, p[clean], o[clean], batch.ii[clean])
        caps = {rid: max(1, int(np.quantile(peaks[:, q], 0.5, method="lower"))) for q, rid in enumerate(packed.resource_ids)}
        problem = with_capacities(problem, caps)
        packed = pack_problem(problem)
        frames_new = FrameSet(packed)  # the same frames, indexed against the new problem tables
        for lanes, sync in frames.frames:
            frames_new.add(lanes, sync)
        frames = frames_new
    return problem, packed, witness, frames, batch, kind
