"""Error types of the batched schedule verifier.

The validation/verification hierarchy has the same names and bases as the
reference's ``src/tilefoundry/schedule/warpgroup/errors.py:6-31`` so callers
that catch ``ValueError`` or the named classes keep working when the GPU
verifier replaces the CPU one.
"""

from __future__ import annotations


class WarpgroupValidationError(ValueError):
    """A typed warpgroup record violates the scheduling contract (errors.py:6)."""


class WarpgroupSerializationError(WarpgroupValidationError):
    """A warpgroup JSON document is malformed or has the wrong format (errors.py:10)."""


class WarpgroupVerificationError(WarpgroupValidationError):
    """A schedule does not satisfy its closed warpgroup problem (errors.py:30)."""


class VerifierRuntimeError(RuntimeError):
    """The native verifier library or the CUDA runtime reported an error."""


class VerifierRangeError(WarpgroupValidationError):
    """A candidate holds a time that the int32 device encoding cannot represent.

    Every materialised start, issue end and completion must lie in
    ``[0, 2**30)``; the reference (unbounded Python ints) has no such limit.
    """


__all__ = [
    "VerifierRangeError",
    "VerifierRuntimeError",
    "WarpgroupSerializationError",
    "WarpgroupValidationError",
    "WarpgroupVerificationError",
]
