"""The C ABI library loads, exports every declared entry point and matches the header's layout.

No GPU is needed: only argument validation that returns before any CUDA call runs.
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from tilefoundry_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tfv.h"


def declared_functions() -> list[str]:
    return re.findall(r"^TFV_API int (tfv_\w+)\(", HEADER.read_text(), flags=re.M)


def test_library_exports_every_declared_function():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.EXPORTS)
    assert lib.tfv_abi_version() == _lib.ABI_VERSION == 5


def test_invalid_arguments_are_rejected_before_cuda():
    lib = _lib.load()
    handle = ctypes.c_void_p()
    assert lib.tfv_problem_create(None, 0, ctypes.byref(handle)) == -1
    desc = _lib.ProblemDesc()
    desc.n_ops = 0
    assert lib.tfv_problem_create(ctypes.byref(desc), 0, ctypes.byref(handle)) == -3
    assert "n_ops" in _lib.last_error()
    import numpy as np

    issue = np.array([1, 1], dtype=np.int32)
    latency = np.array([2, 2], dtype=np.int32)
    wg = np.array([0, 0], dtype=np.int32)
    after = np.array([1, 0], dtype=np.int32)
    before = np.array([0, 1], dtype=np.int32)
    dist = np.array([0, 0], dtype=np.int32)
    desc = _lib.ProblemDesc(2, 3, 1, issue.ctypes.data, latency.ctypes.data, wg.ctypes.data,
                            2, after.ctypes.data, before.ctypes.data, dist.ctypes.data)
    assert lib.tfv_problem_create(ctypes.byref(desc), 0, ctypes.byref(handle)) == -1
    assert "sorted" in _lib.last_error()
    latency[0] = 0
    desc.n_relations = 0
    assert lib.tfv_problem_create(ctypes.byref(desc), 0, ctypes.byref(handle)) == -1
    assert lib.tfv_problem_destroy(None) == 0
    assert lib.tfv_verify_periodic(None, None, None, 0, None, None, None) == -1
    assert lib.tfv_verify_rows(None, None, None, None, None, None) == -1
    assert lib.tfv_analyze_frames(None, None, None, 0, None) == -1
    assert lib.tfv_verify_periodic_host(None, None, None, None) == -1


def test_plan_entry_points_reject_null_before_cuda():
    """The frame-specialised plan entries validate their handles before any CUDA or NVRTC call."""
    lib = _lib.load()
    handle = ctypes.c_void_p()
    options = _lib.PlanOptions(_lib.PLAN_RING, 23, 0)
    assert lib.tfv_plan_create_with(None, None, 0, ctypes.byref(options), ctypes.byref(handle)) == -1
    assert lib.tfv_plan_create(None, None, 0, ctypes.byref(handle)) == -1
    assert lib.tfv_plan_kernel(None) == -1
    assert lib.tfv_plan_delta(None) == -1
    assert lib.tfv_plan_destroy(None) == 0
    buf = ctypes.create_string_buffer(16)
    assert lib.tfv_plan_source(None, buf, len(buf)) == -1
    assert lib.tfv_verify_periodic_planned(None, None, None, 0, None, 0, None, None) == -1
    assert (_lib.PLAN_AUTO, _lib.PLAN_TILES, _lib.PLAN_RING) == (0, 1, 2)


@pytest.mark.parametrize(
    "struct,cname",
    [
        (_lib.ProblemDesc, "tfv_problem_desc"),
        (_lib.Frames, "tfv_frames"),
        (_lib.PeriodicBatch, "tfv_periodic_batch"),
        (_lib.RowsBatch, "tfv_rows_batch"),
        (_lib.Results, "tfv_results"),
        (_lib.PlanOptions, "tfv_plan_options"),
    ],
)
def test_ctypes_layout_matches_header(tmp_path, struct, cname):
    fields = [name for name, _ in struct._fields_]
    body = "\n".join(f'printf("%zu\\n", offsetof({cname}, {f}));' for f in fields)
    src = tmp_path / "layout.c"
    src.write_text(
        f'#include <stddef.h>\n#include <stdio.h>\n#include "tfv.h"\n'
        f'int main(void) {{ printf("%zu\\n", sizeof({cname})); {body} return 0; }}\n'
    )
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    values = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert values[0] == ctypes.sizeof(struct)
    assert values[1:] == [getattr(struct, f).offset for f in fields]
