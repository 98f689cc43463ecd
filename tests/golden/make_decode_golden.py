"""Generate the schedule-document decode fixture from the reference decoder itself.

Run in a container where the reference TileFoundry sources are available:

    python tests/golden/make_decode_golden.py --reference /root/reference

The reference tree is only read; its distribution metadata comes from a temporary
``tilefoundry-0.0.0.dist-info`` (as in make_golden.py). For every golden problem the script
takes schedule documents of its golden raw candidates (serialised as the reference's
schedule format, serialization.py:679-757) plus seeded text mutations of them, runs the
reference's ``warpgroup_schedule_from_json`` (serialization.py:679-727) on each, and writes
``decode_cases.json.gz``:

* ``problem``  — the golden problem each document belongs to;
* ``document`` — the document text;
* ``outcome``  — ``"accepted"``, or the name of the exception class the reference raised;
* ``decoded``  — for accepted documents the decoded record as ``[lanes, sync, rows]``
  (lane operation lists, ``[after, before, distance]`` edges and ``[iteration, operation,
  start, issue_end, completion]`` rows in the record's canonical order), else null.
"""

from __future__ import annotations

import argparse
import gzip
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
TESTS = HERE.parent
SEED = 20261202


def _import_reference(root: Path):
    meta = Path(tempfile.mkdtemp(prefix="tf_meta_"))
    info = meta / "tilefoundry-0.0.0.dist-info"
    info.mkdir()
    (info / "METADATA").write_text("Metadata-Version: 2.1\nName: tilefoundry\nVersion: 0.0.0\n")
    sys.path[:0] = [str(meta), str(root / "src")]
    from tilefoundry.schedule.warpgroup import serialization

    return serialization.warpgroup_schedule_from_json


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", type=Path, required=True, help="root of the reference TileFoundry tree")
    parser.add_argument("--out", type=Path, default=HERE / "decode_cases.json.gz")
    args = parser.parse_args()
    decode = _import_reference(args.reference)
    sys.path[:0] = [str(TESTS), str(TESTS.parent)]
    from golden_data import PROBLEMS, raw_cases
    from test_decode import _document, _mutations

    payload = {"problem": [], "document": [], "outcome": [], "decoded": []}
    for name in PROBLEMS:
        rng = np.random.default_rng(len(name) + SEED)
        cases, _verdicts = raw_cases(name)
        count = 6 if name == "mla" else 40  # the MLA documents are 30 KB each
        base = [_document(*case) for case in cases[:count]]
        docs = base + [m for text in base[: max(2, count // 4)] for m in _mutations(text, rng, 8)]
        for text in docs:
            try:
                record = decode(text)
            except Exception as error:  # the reference's own exception class is the outcome
                payload["problem"].append(name)
                payload["document"].append(text)
                payload["outcome"].append(type(error).__name__)
                payload["decoded"].append(None)
                continue
            payload["problem"].append(name)
            payload["document"].append(text)
            payload["outcome"].append("accepted")
            payload["decoded"].append([
                [list(lane.operations) for lane in record.lanes],
                [[e.after, e.before, e.distance] for e in record.sync],
                [[t.iteration, t.operation_id, t.start, t.issue_end, t.completion] for t in record.times],
            ])
    with gzip.open(args.out, "wt", encoding="utf-8") as handle:
        json.dump(payload, handle, separators=(",", ":"))
    outcomes = {k: payload["outcome"].count(k) for k in sorted(set(payload["outcome"]))}
    print(f"{len(payload['document'])} documents: {outcomes}")


if __name__ == "__main__":
    main()
