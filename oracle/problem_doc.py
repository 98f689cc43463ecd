"""Independent reader of the closed-problem document for the oracle (test infrastructure).

Builds plain namespaces with the attribute names of the reference's
``WarpgroupProblem`` (model.py:377-422) so that :mod:`oracle.verify_port` can run
on fixture problems without the reference or the product package.
"""

from __future__ import annotations

import json
from types import SimpleNamespace


def load_problem(text: str) -> SimpleNamespace:
    doc = json.loads(text)
    ops = []
    for op in doc["loop"]["ops"]:
        ops.append(
            SimpleNamespace(
                id=op["id"],
                warp_group=op["warp_group"],
                issue_duration=op["issue_duration"],
                completion_latency=op["completion_latency"],
                resource_windows=tuple(
                    SimpleNamespace(resource_id=r, amount=a, duration=d) for r, a, d in sorted(map(tuple, op["resource_windows"]))
                ),
                outputs=tuple(
                    SimpleNamespace(id=o["id"], type_id=o["type_id"], expression=ValueUses(tuple(o["uses"])))
                    for o in sorted(op["outputs"], key=lambda item: item["id"])
                ),
            )
        )
    return SimpleNamespace(
        time_unit=doc["time_unit"],
        warp_groups=doc["warp_groups"],
        resources=tuple(SimpleNamespace(id=r["id"], capacity=r["capacity"]) for r in sorted(doc["resources"], key=lambda r: r["id"])),
        types=tuple(SimpleNamespace(id=t["id"], space=t["space"]) for t in doc["types"]),
        inputs=tuple(SimpleNamespace(id=i["id"], type_id=i["type_id"]) for i in doc["inputs"]),
        loop=SimpleNamespace(
            index=doc["loop"]["index"],
            iterations=doc["loop"]["iterations"],
            iter_args=tuple(
                SimpleNamespace(id=a["id"], yield_value=SimpleNamespace(id=a["yield"])) for a in doc["loop"]["iter_args"]
            ),
            ops=tuple(sorted(ops, key=lambda item: item.id)),
        ),
    )


class ValueUses:
    """Expression node listing the SSA values an output reads."""

    __slots__ = ("ids",)

    def __init__(self, ids: tuple[str, ...]) -> None:
        self.ids = ids
