#!/usr/bin/env python
"""Benchmark: candidate schedules verified per second on 1..8 B200 GPUs.

Workload (default ``mla``): seeded neighbourhood perturbations of the MLA decode
example's verified witness schedule (51 operations, 16 iterations, 3 warpgroups, 48
sync edges, 120 required relations), in the compact periodic form (int16 deltas of
the prologue and body-offset starts plus an II and a frame index per candidate). A
step verifies every candidate of one rank's batch: the frame analysis (issued on a side
stream during the previous step's verification, into the second of two frame tables),
the planned call (one preparation launch, the constants kernel and the kernel generated
for the batch's most frequent frame), and for N > 1 the gather of all verdicts to rank 0.

Reported:
  value     whole-job candidates/s with inputs resident in HBM (CUDA events, max over ranks)
  e2e       candidates/s through the C ABI host-buffer entry (tfv_verify_periodic_host):
            pinned host inputs copied in and host results copied out every step
  roofline  the verification kernel's algorithmic bytes per launch / its mean CUDA-event
            duration inside the timed region (events the plan records around the generated
            kernel alone), against the measured HBM copy bandwidth
  cpu_baseline  the oracle (a step-by-step restatement of the reference verifier) on
            all host cores, on a bounded sample of the same batch

``--impl reference`` times that oracle alone (rank 0; other ranks exit at once).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "tests")]

METRIC = "candidate schedules verified/sec (bit-exact verdict+makespan) at 1/2/4/8 B200"
UNIT = "candidates/s"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes per candidate of the MLA batch's default kernel, tfv_spec_ring, measured by ncu
# on a 2 097 152-candidate launch (dram__bytes_read.sum + dram__bytes_write.sum = 444.7 MB +
# 23.5 MB; see profiles/tfv_spec_ring_mla.md). Traffic grows in proportion to the candidates.
MEASURED_DRAM_BYTES_PER_CANDIDATE = (444.7e6 + 23.5e6) / 2097152


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="mla")
    p.add_argument("--candidates", type=int, default=None, help="candidates per GPU (default per workload)")
    p.add_argument("--iis", type=int, default=None,
                   help="initiation intervals per candidate over [II_lb, 2 II_lb] (default 16 for stress, else 1)")
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--e2e-steps", type=int, default=None)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--grouped", action="store_true",
                   help="order the batch by frame (as a search loop emits neighbours variant by variant)")
    p.add_argument("--no-plan", action="store_true",
                   help="skip the kernel generated for the batch's most frequent frame (tfv_plan_create)")
    p.add_argument("--plan-kernel", choices=["auto", "ring", "tiles"], default="auto",
                   help="kernel of the generated plan: ring (producer warp + consumer warps per SM), "
                        "tiles (CTAs in lock step) or auto (the ring when it fits)")
    p.add_argument("--ring-warps", type=int, default=0, help="consumer warps of the ring kernel (0: default)")
    p.add_argument("--no-delta", action="store_true",
                   help="only the plan frame's candidates run the generated code (no delta verification)")
    p.add_argument("--cpu-sample", type=int, default=None, help="oracle sample size per step")
    p.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                   help="N > 1: how each step's packed results reach rank 0: copy engines writing into rank 0's "
                        "memory (peer, shard.PeerGather) or an NCCL gather")
    return p.parse_args()


# --------------------------------------------------------------------------- workload


def mla_workload(n: int, seed: int):
    from golden_data import problem_text, raw_cases
    from tilefoundry_b200 import pack_problem, problem_from_json
    from tilefoundry_b200.workloads import mla_perturbations, shared_producers, witness_from_rows

    problem = problem_from_json(problem_text("mla"))
    packed = pack_problem(problem)
    witness = witness_from_rows(packed, *raw_cases("mla")[0][0])
    frames, batch, _kind = mla_perturbations(packed, witness, n, seed=seed, producers=shared_producers(problem))
    return problem, packed, frames, batch


def body_workload(name: str):
    def make(n: int, seed: int):
        from tilefoundry_b200.workloads import body_batch

        problem, packed, _witness, frames, batch, _kind = body_batch(name, n, seed=seed)
        return problem, packed, frames, batch

    return make


# name: (generator, default candidates per GPU, description). The kernel bodies' candidates
# are software-pipelined schedules of the body, half of them corrupted (workloads.body_batch).
WORKLOADS = {
    "mla": (mla_workload, 1 << 23, "mla-decode-perturbations"),
    "gemm": (body_workload("gemm"), 1 << 22, "gemm-mainloop-pipelined"),
    "fa": (body_workload("fa"), 1 << 22, "flash-attention-fwd-pipelined"),
    "dag": (body_workload("dag"), 1 << 21, "layered-dag-256-pipelined"),
    "stress": (body_workload("stress"), 1 << 16, "stress-dag-1024-pipelined"),
}
# Bodies of this many operations or more run the large-body kernel (one warp per candidate);
# smaller ones the kernel generated for the batch's most frequent frame.
LARGE_MIN_OPS = 128


def workload(name: str, n: int, seed: int):
    return WORKLOADS[name][0](n, seed)


def algorithmic_bytes_per_candidate(n_ops: int) -> int:
    """Inputs: int16 prologue and offset deltas per op, int32 II and frame; outputs: 3 x int32."""
    return 2 * 2 * n_ops + 4 + 4 + 12


def workload_config(args, packed, frames, n: int, n_ii: int, world: int) -> dict:
    """The workload description both arms print (the same dict for the same arguments)."""
    per_launch = (algorithmic_bytes_per_candidate(packed.n_ops) + 16 * (n_ii - 1)) * n
    return {
        "workload": WORKLOADS[args.workload][2],
        "candidates_per_gpu": n,
        "iis_per_candidate": n_ii,
        "ops": packed.n_ops,
        "iterations": packed.iterations,
        "warpgroups": packed.warp_groups,
        "relations": int(packed.relations.shape[0]),
        "frames": len(frames),
        "format": "periodic: int16 prologue/offset deltas + int32 ii + int32 frame per candidate",
        "bytes_per_candidate": algorithmic_bytes_per_candidate(packed.n_ops),
        "l2": f"inputs {per_launch / 1e9:.2f} GB per GPU per step, larger than the 126 MB L2",
        "parallelism": f"dp{world} (contiguous candidate shards; int8 verdict + int32 makespan gathered to rank 0"
                       + (f", {args.gather})" if world > 1 else ")"),
    }


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), or the platform's processor string."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def default_iis(args) -> int:
    return args.iis or (16 if args.workload == "stress" else 1)


# --------------------------------------------------------------------------- oracle timing


ORACLE_PROBLEM = None  # closed-problem JSON text of the workload, set before the pool starts


def _oracle_worker(args):
    text, chunk = args
    from oracle import verify_port as port
    from oracle.problem_doc import load_problem

    problem = load_problem(text)
    return [port.classify(problem, *case)[0] for case in chunk]


def oracle_sample(frames, batch, packed, start: int, count: int):
    """Raw (lanes, sync, rows) candidates [start, start + count) of a periodic batch."""
    import numpy as np

    cases = []
    n = batch.n
    for j in range(count):
        c = (start + j) % n
        lanes, sync = frames.frames[int(batch.frame[c])]
        p = batch.base_prologue.astype(np.int64) + batch.prologue_delta[:, c].astype(np.int64)
        o = batch.base_offset.astype(np.int64) + batch.offset_delta[:, c].astype(np.int64)
        ii = int(batch.ii[c])
        rows = []
        for i in range(packed.iterations):
            for k, op in enumerate(packed.op_ids):
                s = int(p[k]) if i == 0 else int(o[k]) + i * ii
                rows.append((i, op, s, s + int(packed.issue[k]), s + int(packed.latency[k])))
        cases.append(([list(l) for l in lanes], [tuple(e) for e in sync], rows))
    return cases


def time_oracle(pool, workers: int, frames, batch, packed, start: int, count: int) -> float:
    cases = oracle_sample(frames, batch, packed, start, count)
    chunks = [cases[k::workers] for k in range(workers)]
    t0 = time.perf_counter()
    list(pool.map(_oracle_worker, [(ORACLE_PROBLEM, chunk) for chunk in chunks if chunk]))
    return time.perf_counter() - t0


def make_pool():
    import multiprocessing as mp
    from concurrent.futures import ProcessPoolExecutor

    workers = os.cpu_count() or 1
    return ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn")), workers


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    pool, workers = make_pool()
    global ORACLE_PROBLEM
    n = args.candidates or WORKLOADS[args.workload][1]  # the GPU arm's batch (rank 0's seed)
    problem, packed, frames, batch = workload(args.workload, n, args.seed)
    from tilefoundry_b200 import problem_to_json

    ORACLE_PROBLEM = problem_to_json(problem)
    sample = args.cpu_sample or max(16, 4 * workers)
    with pool:
        for w in range(args.warmup):
            time_oracle(pool, workers, frames, batch, packed, w, min(workers, 8))
        total, elapsed = 0, 0.0
        for s in range(args.steps):
            elapsed += time_oracle(pool, workers, frames, batch, packed, 1000 + s * sample, sample)
            total += sample
    value = total / elapsed
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * elapsed / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int64",
        "data": "synthetic: seeded candidates of the workload (same generator and seed as the GPU arm)",
        "config": workload_config(args, packed, frames, n, default_iis(args), int(os.environ.get("WORLD_SIZE", "1"))),
        "cpu_baseline": {
            "value": value,
            "unit": UNIT,
            "cores": workers,
            "cpu_model": cpu_model(),
            "kind": "port",
            "sample": f"{sample} candidates per step of this batch (each at its own II), {args.steps} steps, "
                      f"oracle/verify_port.py in {workers} processes",
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- clocks


class ClockSampler:
    """Polls NVML (read-only) for SM clock and clock-event reasons while running."""

    REASONS = {
        "gpu_idle": 0x1,
        "applications_clocks_setting": 0x2,
        "sw_power_cap": 0x4,
        "hw_slowdown": 0x8,
        "sync_boost": 0x10,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, torch_device: int) -> None:
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(torch_device)
            want = (int(props.pci_domain_id), int(props.pci_bus_id), int(props.pci_device_id))
            handle = None
            for k in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(k)
                info = pynvml.nvmlDeviceGetPciInfo(h)
                if (int(info.domain), int(info.bus), int(info.device)) == want:
                    handle = h
            self._nvml = pynvml
            self._handle = handle
            if handle is not None:
                self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._handle = None

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = set()
        for _, bits in self.samples:
            for name, bit in self.REASONS.items():
                if bits & bit and name != "gpu_idle":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(m for m, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(reasons),
            "samples": len(self.samples),
        }


# --------------------------------------------------------------------------- GPU arm


def link_bandwidth(device: int, nbytes: int = 1 << 29) -> dict:
    """Pinned host <-> device copy bandwidth of this GPU (CUDA events, best of 3) and the
    NUMA node its PCI device sits on; they bound the host-buffer entry."""
    import torch

    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dev = torch.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", device))
    stream = torch.cuda.current_stream(device)
    rates = {}
    for name, (dst, src) in {"h2d_gbs": (dev, host), "d2h_gbs": (host, dev)}.items():
        best = float("inf")
        for _ in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dst.copy_(src, non_blocking=True)
            b.record(stream)
            b.synchronize()
            best = min(best, a.elapsed_time(b))
        rates[name] = nbytes / (best / 1e3) / 1e9
    props = torch.cuda.get_device_properties(device)
    bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    try:
        numa = int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text().strip())
    except (OSError, ValueError):
        numa = None
    del host, dev
    return {**rates, "gpu_pci": bus, "gpu_numa_node": numa, "host_cpus": len(os.sched_getaffinity(0))}


def run_ours(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    want_cpu = world == 1 and rank == 0 and not args.no_cpu_baseline and args.workload in ("mla", "gemm", "fa")
    pool, workers = make_pool() if want_cpu else (None, 0)  # spawned before any CUDA call

    import numpy as np
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from tilefoundry_b200 import VerifierRuntimeError, WarpgroupVerifier
    from tilefoundry_b200.verify import pinned_like

    global ORACLE_PROBLEM
    n = args.candidates or WORKLOADS[args.workload][1]
    n_ii = default_iis(args)
    problem, packed, frames, batch = workload(args.workload, n, args.seed + rank)
    if args.grouped:  # same candidates, frame by frame
        from tilefoundry_b200.batch import PeriodicBatch

        order = np.argsort(batch.frame, kind="stable")
        batch = PeriodicBatch(batch.base_prologue, batch.base_offset,
                              np.ascontiguousarray(batch.prologue_delta[:, order]),
                              np.ascontiguousarray(batch.offset_delta[:, order]), batch.ii[order], batch.frame[order])
    from tilefoundry_b200 import problem_to_json

    ORACLE_PROBLEM = problem_to_json(problem)
    verifier = WarpgroupVerifier(packed, device=local)
    dframes = verifier.frames_to_device(frames)
    tensors = {
        key: torch.from_numpy(np.ascontiguousarray(getattr(batch, key))).to(dev)
        for key in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")
    }
    # Results, double-buffered so that the gather of one step's results to rank 0 overlaps
    # the next step's verification: int32 verdict and II [n_ii, n], and the gathered
    # payload (shard.pack_results: int32 makespans, written there by the verifier, then
    # int8 verdicts; 5 bytes per schedule). With n_ii > 1 every candidate is verified at
    # n_ii IIs spread over [II_lb, 2 II_lb].
    from tilefoundry_b200.shard import pack_results
    from tilefoundry_b200.workloads import ii_lower_bound, ii_sweep

    sweep = np.repeat(ii_sweep(ii_lower_bound(packed), n_ii)[:, None], n, axis=1).astype(np.int32) if n_ii > 1 else None
    ii_values = torch.from_numpy(sweep).to(dev) if sweep is not None else None
    m = n_ii * n
    verdicts = [torch.empty((n_ii, n), dtype=torch.int32, device=dev) for _ in range(2)]
    iis = [torch.empty((n_ii, n), dtype=torch.int32, device=dev) for _ in range(2)]
    payload = [torch.empty(5 * m, dtype=torch.uint8, device=dev) for _ in range(2)]
    makespans = [buf[: 4 * m].view(torch.int32).view(n_ii, n) for buf in payload]
    peer = None
    if world > 1 and args.gather == "peer":
        from tilefoundry_b200.shard import PeerGather

        peer = PeerGather(5 * m)
    gathered = [[torch.empty(5 * m, dtype=torch.uint8, device=dev) for _ in range(world)] if rank == 0 else None
                for _ in range(2)] if world > 1 and peer is None else None
    pending = [None, None]
    # Two frame tables: the analysis of step s + 1's frames runs on a side stream while step s
    # verifies (its one-warp CTAs fit beside the ring kernel's on every SM), into the table
    # step s - 1 used; each step's verification waits for its own table's analysis.
    tables = [verifier.analyze(dframes), verifier.analyze(dframes)]
    stream = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    analysed = [torch.cuda.Event() for _ in range(2)]
    released = [None, None]  # per table: an event after the last call that read it
    # The batch's most frequent frame gets a kernel generated and compiled for it (before
    # any timing); its candidates run that code, the others the frame-table path.
    plan, spec_frame, plan_compile_ms = None, -1, None
    if not args.no_plan and n_ii == 1 and packed.n_ops < LARGE_MIN_OPS:
        spec_frame = int(np.argmax(np.bincount(batch.frame, minlength=len(frames))))
        t0 = time.perf_counter()
        try:
            plan = verifier.plan(frames, spec_frame, kernel=args.plan_kernel, ring_warps=args.ring_warps,
                                 delta=not args.no_delta)
            plan_compile_ms = 1000.0 * (time.perf_counter() - t0)  # NVRTC compile + module load, once per frame
        except VerifierRuntimeError as error:  # no run-time compiler here: the frame-table kernel serves all
            print(f"# frame-specialised kernel unavailable ({error}); frame-table kernel only", file=sys.stderr)
            plan, spec_frame = None, -1

    def barrier():
        if dist is not None:
            dist.barrier()

    def analyse(s, events=None):
        """Issue the frame analysis of step s into table s % 2 on the side stream."""
        k = s % 2
        if released[k] is not None:
            side.wait_event(released[k])
        if events is not None:
            events[0].record(side)
        verifier.analyze(dframes, table=tables[k], stream=side)
        if events is not None:
            events[1].record(side)
        analysed[k].record(side)

    def step(s, events=None, next_events=None):
        """Verify step s (its analysis already issued); then issue step s + 1's analysis
        unless next_events is False (the last step)."""
        buf = s % 2
        if peer is not None:
            peer.wait(buf, stream)  # the stream waits until that copy has read the buffer
        if pending[buf] is not None:
            pending[buf].wait()  # the stream waits until that gather has read the buffer
            pending[buf] = None
        stream.wait_event(analysed[s % 2])
        if events is not None:
            events[2].record(stream)
        out = (verdicts[buf], makespans[buf], iis[buf])
        if ii_values is None:
            verifier.verify_periodic_device(dframes, tables[s % 2], tensors, out=tuple(t[0] for t in out),
                                            plan=plan, spec_frame=spec_frame)
        else:
            verifier.verify_periodic_sweep_device(dframes, tables[s % 2], tensors, ii_values, out=out)
        if events is not None:
            events[3].record(stream)
        released[s % 2] = torch.cuda.Event()
        released[s % 2].record(stream)
        if next_events is not False:
            analyse(s + 1, next_events)
        if dist is not None:
            pack_results(verdicts[buf], makespans[buf], out=payload[buf])
            if peer is not None:
                peer.send(buf, payload[buf], stream)
            else:
                pending[buf] = dist.gather(payload[buf], gather_list=gathered[buf] if rank == 0 else None, dst=0,
                                           async_op=True)

    def drain():
        if peer is not None:
            stream.wait_stream(peer.stream)  # the copies are part of the step
        for k in range(2):
            if pending[k] is not None:
                pending[k].wait()
                pending[k] = None

    analyse(0)
    for s in range(args.warmup):
        step(s, next_events=None if s + 1 < args.warmup else False)
    drain()
    torch.cuda.synchronize(dev)
    barrier()
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    begin = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if plan is not None:  # CUDA events around the generated kernel alone, recorded by the plan
        plan.kernel_times()
        plan.set_timing(True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize(dev)
        barrier()
        begin.record(stream)
        side.wait_stream(stream)  # the first analysis starts inside the timed region
        analyse(0, events[0])
        for s in range(args.steps):
            step(s, events[s], events[s + 1] if s + 1 < args.steps else False)
        drain()
        end.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
    elapsed_ms = begin.elapsed_time(end)
    plan_kernel_ms = None
    if plan is not None:
        plan.set_timing(False)
        plan_kernel_ms = plan.kernel_times()
        assert len(plan_kernel_ms) == args.steps, "one timed generated kernel per step"
    if peer is not None:  # every rank's last payload arrived intact in rank 0's memory
        last_buf = (args.steps - 1) % 2
        mine = int(payload[last_buf].to(torch.int64).sum().item())
        sums = [None] * world
        dist.all_gather_object(sums, mine)
        if rank == 0:
            rows = peer.received(last_buf).to(torch.int64).sum(dim=1).tolist()
            assert rows == sums, "peer gather rows differ from the ranks' payloads"
    analyze_ms = [e[0].elapsed_time(e[1]) for e in events]
    verify_ms = [e[2].elapsed_time(e[3]) for e in events]
    per_rank = None
    if dist is not None:
        # every rank's step time, generated-kernel time and call time (diagnostics), then the max
        mine = torch.tensor([elapsed_ms / args.steps,
                             statistics.mean(plan_kernel_ms) if plan_kernel_ms else float("nan"),
                             statistics.mean(verify_ms)], device=dev, dtype=torch.float64)
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        per_rank = {key: [round(float(t[i].item()), 4) for t in every]
                    for i, key in enumerate(("ms_per_step", "kernel_ms", "call_ms"))}
        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    value = n * n_ii * world * args.steps / (elapsed_ms / 1e3)

    # End to end through the C ABI host-buffer entry: pinned inputs in, host results out.
    from tilefoundry_b200.batch import PeriodicBatch

    hb = PeriodicBatch(*(pinned_like(getattr(batch, key)) for key in (
        "base_prologue", "base_offset", "prologue_delta", "offset_delta", "ii", "frame")))
    host_out = tuple(pinned_like(np.empty(n, dtype=np.int32)) for _ in range(3))
    arrays = frames.arrays()
    from tilefoundry_b200 import _lib

    fstruct = _lib.frames_struct(arrays, len(frames))
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 10))
    if sweep is None:
        def e2e_call():
            verifier.verify_periodic_host_arrays(fstruct, hb, host_out)
            return host_out
        e2e_entry = "tfv_verify_periodic_host"
    else:
        def e2e_call():  # host arrays in, host arrays out, through the public sweep entry
            return verifier.verify_periodic_sweep(frames, hb, sweep)
        e2e_entry = "WarpgroupVerifier.verify_periodic_sweep"
    for _ in range(min(args.warmup, 2)):
        e2e_call()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_out = e2e_call()
    e2e_s = time.perf_counter() - t0
    barrier()
    if dist is not None:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = n * n_ii * world * e2e_steps / e2e_s
    last = verdicts[(args.steps - 1) % 2]
    assert np.array_equal(np.asarray(e2e_out[0]).reshape(n_ii, n), last.cpu().numpy()), \
        "host-buffer and device entries disagree"
    link = link_bandwidth(local)
    h2d = sum(int(np.asarray(v).nbytes) for v in arrays.values()) + sum(
        int(getattr(batch, k).nbytes) for k in ("base_prologue", "base_offset", "prologue_delta", "offset_delta", "frame"))
    h2d += int(sweep.nbytes) if sweep is not None else int(batch.ii.nbytes)
    d2h = 3 * 4 * n * n_ii

    if rank == 0:
        # deltas and frame once per candidate; II and the three results once per (candidate, II)
        per_launch = (algorithmic_bytes_per_candidate(packed.n_ops) + 16 * (n_ii - 1)) * n
        # the dominant kernel's own launches: the generated kernel (events the plan records
        # around it), else the whole verify call (one verification kernel and the small
        # sync-program kernel before it)
        kernel_ms = statistics.mean(plan_kernel_ms) if plan_kernel_ms else statistics.mean(verify_ms)
        achieved = per_launch / (kernel_ms / 1e3) / 1e9
        peak, peak_src = FALLBACK_HBM_GBS, "fallback"
        peaks = ROOT / "MEASURED_PEAKS.json"
        if peaks.exists():
            peak, peak_src = float(json.loads(peaks.read_text())["hbm_gbs"]), "measured"
        cpu = None
        if want_cpu:
            sample = args.cpu_sample or max(16, 4 * workers)
            with pool:
                time_oracle(pool, workers, frames, batch, packed, 0, min(workers, 8))
                secs = time_oracle(pool, workers, frames, batch, packed, 7, sample)
            cpu = {
                "value": sample / secs,
                "unit": UNIT,
                "cores": workers,
                "cpu_model": cpu_model(),
                "kind": "port",
                "sample": f"{sample} candidates of this batch through oracle/verify_port.py in {workers} processes ({secs:.1f} s)",
            }
        histogram = np.bincount(last.cpu().numpy().ravel() + 4, minlength=26)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int32",
            "data": ("synthetic: seeded perturbations of the MLA example's verified witness (per-rank seed)"
                     if args.workload == "mla" else
                     "synthetic: seeded software-pipelined schedules of the body, half corrupted (per-rank seed)"),
            "config": workload_config(args, packed, frames, n, n_ii, world),
            "valid_fraction": float(histogram[4] / (n * n_ii)),
            "plan": None if plan is None else {
                "kernel": plan.kernel, "delta": plan.delta, "ring_warps": plan.ring_warps,
                "compile_ms": plan_compile_ms,
                "note": "compiled once per frame content before timing; a share of "
                        f"{plan_compile_ms / (plan_compile_ms + elapsed_ms):.3f} of compile + timed region",
            },
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": MEASURED_DRAM_BYTES_PER_CANDIDATE * n if args.workload == "mla" else None,
                "traffic_source": "ncu dram__bytes_read+write of tfv_spec_ring on 2097152 MLA candidates, "
                                  "scaled per candidate" if args.workload == "mla" else None,
                "peak_source": peak_src,
                "kernel": (("tfv_spec_ring" if plan.kernel == "ring" else "tfv_spec_kernel") +
                           " (generated for the most frequent frame, "
                           f"{float(np.mean(batch.frame == spec_frame)):.2f} of the batch)" if plan is not None else
                           "tfv::verify_periodic_large_kernel" if packed.n_ops >= LARGE_MIN_OPS else
                           "tfv::verify_periodic_tma_kernel"),
                "kernel_ms": kernel_ms,
                "kernel_timing": ("CUDA events recorded by the plan on the call's stream around the generated "
                                  "kernel's launch" if plan_kernel_ms else
                                  "CUDA events around the verify call on its stream"),
                "call_ms": statistics.mean(verify_ms),
                "analyze_ms": statistics.mean(analyze_ms),
            },
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps, "entry": e2e_entry, **link,
                    # the copies bound the entry: one step of a rank needs h2d / h2d_gbs + d2h /
                    # d2h_gbs on its GPU's host link (rank 0's link measured, every rank has its own)
                    "link_bound": world * n * n_ii / (h2d / (link["h2d_gbs"] * 1e9) + d2h / (link["d2h_gbs"] * 1e9)),
                    "frac_of_link_bound": e2e_value / (world * n * n_ii / (h2d / (link["h2d_gbs"] * 1e9) +
                                                                           d2h / (link["d2h_gbs"] * 1e9)))},
            # per step: the frame analysis, then either the sync-program compile and the
            # verification kernel, or the plan's preparation (spec-frame check, sync programs,
            # frame comparison in one launch), constants kernel and generated kernel
            "gpu_launches": (3 if plan is None else 4) * args.steps,
            "ranks": per_rank,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    verifier.close()
    if dist is not None:
        dist.barrier()
        if peer is not None:  # the other ranks unmap rank 0's buffers before rank 0 frees them
            if rank != 0:
                peer.close()
            dist.barrier()
            if rank == 0:
                peer.close()
        dist.destroy_process_group()


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
