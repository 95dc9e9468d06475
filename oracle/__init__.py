"""ORACLE — test infrastructure only.

A CPU restatement, in plain PyTorch-on-CPU arithmetic, of the reference algorithms on invokerl's
training hot path (the reference itself is pure Python over PyTorch).  It is the checker for the
CUDA kernels: only the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg and
reference arm may import it.  The product package ``invokerl_b200`` never imports it and has no
CPU path of its own.

Parity pin: the functions here are checked against golden vectors produced by running the
reference's own code (``invokerl`` at the pinned commit) on seeded inputs; see
``tests/golden/make_golden.py`` and ``tests/test_oracle_golden.py``.
"""

from .reference_math import *  # noqa: F401,F403
