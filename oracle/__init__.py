"""CPU oracle for the V1 query-side selection path (test infrastructure only).

This package restates the reference algorithms in numpy so that the CUDA
kernels in the product can be checked against them.  It is imported only by
``tests/``, by ``__graft_entry__.smoke()`` (as the checker) and by
``bench.py``'s CPU-baseline / ``--impl reference`` legs.  The product package
never imports it and never falls back to it.
"""
from .v1x_oracle import *  # noqa: F401,F403
