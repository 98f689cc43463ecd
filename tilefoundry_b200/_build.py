"""Compile the native verifier library ``libtfv.so`` in-tree for sm_100a.

The library is built from ``csrc/*.cu`` with nvcc (``-gencode
arch=compute_100a,code=sm_100a``) and placed next to this file, where
``tilefoundry_b200._lib`` loads it. The CUDA runtime is linked statically so the
library does not depend on the runtime version that PyTorch bundles.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
SOURCES = sorted((PACKAGE / "csrc").glob("*.cu"))
HEADERS = sorted((PACKAGE / "csrc").glob("*.cuh")) + [ROOT / "include" / "tfv.h"]
LIBRARY = PACKAGE / "libtfv.so"

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O2,-fvisibility=hidden",
    "-shared",
    "-cudart",
    "static",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; install the CUDA toolkit to build libtfv.so")
    return found


def is_stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    return any(path.stat().st_mtime > built for path in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Build ``libtfv.so`` unless it is newer than every source and header."""
    if not force and not is_stale():
        return LIBRARY
    tmp = LIBRARY.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-I", str(PACKAGE / "csrc"), *map(str, SOURCES), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr}")
    os.replace(tmp, LIBRARY)
    if verbose:
        print(result.stderr)
    return LIBRARY


if __name__ == "__main__":
    build(force=True, verbose=True)
