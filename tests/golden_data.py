"""Loaders for the committed golden fixtures (tests/golden/, made by make_golden.py)."""

from __future__ import annotations

import gzip
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
PROBLEMS = sorted(p.name[: -len("_problem.json")] for p in GOLDEN.glob("*_problem.json"))


def problem_text(name: str) -> str:
    return (GOLDEN / f"{name}_problem.json").read_text(encoding="utf-8")


def raw_cases(name: str):
    """[(lanes, sync, rows)], [(class, makespan, ii)] with rows as tuples."""
    with gzip.open(GOLDEN / f"{name}_raw.json.gz", "rt", encoding="utf-8") as handle:
        payload = json.load(handle)
    cases = [
        ([list(lane) for lane in lanes], [tuple(e) for e in sync], [tuple(r) for r in rows])
        for lanes, sync, rows in payload["candidates"]
    ]
    return cases, [tuple(v) for v in payload["verdicts"]]


def periodic_cases(name: str) -> dict:
    data = np.load(GOLDEN / f"{name}_periodic.npz")
    frames = [(lanes, [tuple(e) for e in sync]) for lanes, sync in json.loads(str(data["frames"]))]
    return {
        "frames": frames,
        "prologue": data["prologue"].astype(np.int64),
        "offset": data["offset"].astype(np.int64),
        "ii": data["ii"].astype(np.int64),
        "frame": data["frame"].astype(np.int64),
        "verdict": data["verdict"].astype(np.int64),
        "makespan": data["makespan"].astype(np.int64),
        "iiv": data["iiv"].astype(np.int64),
    }
