"""The reference's own record types, where the reference package is installed.

``baseline/_ref`` holds the reference TileFoundry package when it was installed there (the
offline ``pip install --target baseline/_ref`` of the reference tree); without it these
helpers report it unavailable and the tests that use them skip. Problems are rebuilt as the
reference's ``WarpgroupProblem`` records (model.py:377) from the golden closed-problem
documents: every output's expression references exactly the values the document lists (a
copy of one value, an elementwise sum of several, a scalar literal of none), which is all the
verifier reads of an expression (verify.py:32-52 through value_references).
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def available() -> bool:
    return (REF_ROOT / "tilefoundry" / "schedule" / "warpgroup" / "model.py").is_file()


def modules():
    """``(model, expression, errors)`` modules of the reference package."""
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    from tilefoundry.schedule.warpgroup import errors, expression, model

    return model, expression, errors


def problem(text: str):
    """The reference WarpgroupProblem of a closed-problem document."""
    m, e, _ = modules()
    d = json.loads(text)
    types = tuple(m.TensorType(t["id"], (1,), m.DType("fp32"), m.MemorySpace(t["space"])) for t in d["types"])
    inputs = tuple(m.ProgramInput(i["id"], i["type_id"]) for i in d["inputs"])

    def expression(uses):
        refs = tuple(e.ValueRef(u) for u in uses)
        if not refs:
            return e.ScalarLiteral(0.0)
        if len(refs) == 1:
            return e.CopyExpression(refs[0])
        return e.ElementwiseExpression(e.ElementwiseOperator.ADD, refs)

    loop = d["loop"]
    iter_args = tuple(m.LoopIterArg(a["id"], e.ScalarLiteral(0), e.ValueRef(a["yield"])) for a in loop["iter_args"])
    ops = tuple(
        m.ProblemOperation(
            o["id"],
            tuple(m.OperationOutput(x["id"], x["type_id"], expression(x["uses"])) for x in o["outputs"]),
            o["warp_group"], o["issue_duration"], o["completion_latency"],
            tuple(m.ResourceWindow(*w) for w in o["resource_windows"]),
        )
        for o in loop["ops"]
    )
    return m.WarpgroupProblem(
        d["time_unit"], d["warp_groups"], tuple(m.ResourceCapacity(r["id"], r["capacity"]) for r in d["resources"]),
        types, inputs, m.ProblemLoop(loop["index"], loop["iterations"], iter_args, ops),
    )


def schedule(lanes, sync, rows):
    """The reference WarpgroupSchedule of a raw candidate, or None where its constructors
    refuse it (the candidate's verdict is then class 1)."""
    m, _, errors = modules()
    try:
        return m.WarpgroupSchedule(
            m.SCHEDULE_FORMAT,
            tuple(m.WarpgroupLane(tuple(lane)) for lane in lanes),
            tuple(m.SynchronizationEdge(*edge) for edge in sync),
            tuple(m.TimedOperation(*row) for row in rows),
        )
    except (errors.WarpgroupValidationError, TypeError, ValueError):
        return None
