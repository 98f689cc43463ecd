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


__all__ = ["MIX", "Witness", "absolute_starts", "mla_perturbations", "shared_producers", "witness_from_rows"]


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
        ProblemLoop("%k", iterations, tuple(LoopIterArg(a, ValueRef(y)) for a, y in iter_args), ops),
    )


def gemm_mainloop_problem(iterations: int = 8):
    """GEMM mainloop body: TMA loads of A (128x64 bf16, 16 KB) and B (256x64 bf16, 32 KB)
    by the producer warpgroup, a 128x256x64 tcgen05 MMA (latency 512) and a barrier
    arrive by the consumer, and an epilogue store of the 128x256 fp32 accumulator.
    Resources: shared memory in KB (227), TMEM columns (512), mbarriers, TMA slots; a
    4-stage ring bounds the loads in flight through the TMA-slot capacity."""
    spec = [
        ("load_a", 0, 24, 700, [("smem_kb", 16, 700), ("tma_slots", 1, 700)], "%a", "shared", ["%gmem"]),
        ("load_b", 0, 24, 900, [("smem_kb", 32, 900), ("tma_slots", 1, 900)], "%b", "shared", ["%gmem"]),
        ("mma", 1, 64, 512, [("tmem_cols", 256, 512)], "%acc", "shared", ["%a", "%b", "%acc_prev"]),
        ("arrive", 1, 4, 4, [("mbarrier", 1, 4)], "%bar", "register", ["%acc"]),
        ("store", 1, 160, 420, [("smem_kb", 96, 420)], "%out", "register", ["%acc", "%bar"]),
    ]
    caps = {"smem_kb": 227, "tmem_cols": 512, "mbarrier": 8, "tma_slots": 8}
    return _body_problem(spec, 2, iterations, caps, iter_args=[("%acc_prev", "%acc")])


def flash_attention_problem(iterations: int = 16):
    """FlashAttention-forward body (Q 128x128, K/V 128x128 bf16 tiles): loads of K and V
    (load warpgroup), S = QK^T and P.V MMAs (MMA warpgroup), rowmax, exp2, rowsum and the O
    rescale (softmax warpgroup). Shared memory 227 KB, TMEM 512 columns."""
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
