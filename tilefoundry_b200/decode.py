"""Native decode of schedule documents straight into the packed rows layout.

``decode_schedule_documents`` hands a batch of schedule JSON documents to
``tfv_decode_schedules`` (host code in ``libtfv.so``, several threads), which applies
the reference's strict JSON rules and record constructors (serialization.py:679-727,
model.py:425-507) and writes dense timing rows and deduplicated frames in the layout
the rows kernel reads. It produces the same arrays as ``schedule_from_json`` followed
by ``pack_rows``, without building Python records.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import numpy as np

from . import _lib
from .batch import RowsBatch
from .problem import PackedProblem

#: Verdict of a document that does not decode (the reference raises
#: WarpgroupSerializationError before verifying it).
CLASS_DECODE_FAILED = -4


class NativeFrameSet:
    """A ``tfv_frameset``: frames deduplicated across every decode into it."""

    def __init__(self, packed: PackedProblem) -> None:
        self._lib = _lib.load()
        self.packed = packed
        ids = (ctypes.c_char_p * max(1, packed.n_ops))(*(op.encode("ascii") for op in packed.op_ids))
        handle = ctypes.c_void_p()
        _lib.check(self._lib.tfv_frameset_create(packed.n_ops, packed.iterations, ids, ctypes.byref(handle)),
                   "tfv_frameset_create")
        self._handle = handle

    def close(self) -> None:
        if self._handle:
            self._lib.tfv_frameset_destroy(self._handle)
            self._handle = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        try:
            self.close()
        except Exception:
            pass

    def struct(self) -> _lib.Frames:
        """Host view in the layout of ``tfv_frames`` (valid until the next decode)."""
        view = _lib.Frames()
        _lib.check(self._lib.tfv_frameset_view(self._handle, ctypes.byref(view)), "tfv_frameset_view")
        return view

    def arrays(self) -> dict[str, np.ndarray]:
        """Copies of the frame arrays (same keys as ``FrameSet.arrays``)."""
        v = self.struct()
        n, N = v.n_frames, self.packed.n_ops
        S, E = v.n_sync_sets, v.n_sync_edges

        def take(ptr, count, ctype, dtype):
            if count == 0:
                return np.zeros(0, dtype=dtype)
            return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctype)), shape=(count,)).astype(dtype)

        edges = take(v.sync_edges, 3 * E, ctypes.c_int32, np.int32).reshape(-1, 3)
        return {
            "lane_pos": take(v.lane_pos, n * N, ctypes.c_uint16, np.uint16).reshape(n, N),
            "lane_count": take(v.lane_count, n, ctypes.c_int32, np.int32),
            "flags": take(v.flags, n, ctypes.c_int32, np.int32),
            "sync_set": take(v.sync_set, n, ctypes.c_int32, np.int32),
            "sync_offsets": take(v.sync_offsets, S + 1, ctypes.c_int32, np.int32),
            "sync_edges": edges if edges.size else np.zeros((1, 3), dtype=np.int32),
        }

    def __len__(self) -> int:
        return int(self.struct().n_frames)


@dataclass
class DecodedBatch:
    rows: RowsBatch
    status: np.ndarray  # [n] int32: 0 decoded, 1 rejected like WarpgroupSerializationError


def decode_schedule_documents(frames: NativeFrameSet, documents: Sequence[str | bytes], *, threads: int = 0) -> DecodedBatch:
    """Decode ``documents`` into rows (and frames of ``frames``)."""
    packed = frames.packed
    n, N, I = len(documents), packed.n_ops, packed.iterations
    blobs = [d.encode("utf-8") if isinstance(d, str) else bytes(d) for d in documents]
    texts = (ctypes.c_char_p * max(1, n))(*blobs)
    lengths = (ctypes.c_size_t * max(1, n))(*(len(b) for b in blobs))
    start = np.empty((n, I, N), dtype=np.int32)
    issue_end = np.empty((n, I, N), dtype=np.int32)
    completion = np.empty((n, I, N), dtype=np.int32)
    frame, flags, mk, ii, status = (np.empty(n, dtype=np.int32) for _ in range(5))
    p = lambda a: a.ctypes.data  # noqa: E731
    _lib.check(
        frames._lib.tfv_decode_schedules(frames._handle, n, texts, lengths, p(start), p(issue_end), p(completion),
                                         p(frame), p(flags), p(mk), p(ii), p(status), threads),
        "tfv_decode_schedules",
    )
    rows = RowsBatch(start, issue_end, completion, frame, flags, flags != 0, mk, ii)
    return DecodedBatch(rows, status)


__all__ = ["CLASS_DECODE_FAILED", "DecodedBatch", "NativeFrameSet", "decode_schedule_documents"]
