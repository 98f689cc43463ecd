"""CPU oracle of the schedule verifier: test infrastructure, never a product code path.

* :mod:`oracle.verify_port` — step-by-step Python restatement of the reference
  verifier (``verify.py``) and its record constructors.
* :mod:`oracle.fast` — batch driver for ``tfv_oracle.c``, the same restatement in C.
"""
