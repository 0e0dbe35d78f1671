"""CPU oracle for the spTiles hot path -- TEST INFRASTRUCTURE ONLY.

This package restates the arithmetic of the reference's SPIR-V shaders
(src/tileops.hpp) on the CPU.  It is the checker: only the test suite, the
smoke check and the benchmark's CPU-baseline leg import it.  The product
(`sptiles_b200`) never does.

Parity pin: checked against the reference's own known-answer tests through
the golden fixtures under tests/golden (generated from the reference's Python
code by tests/golden/make_golden.py).
"""
from .oracle import *  # noqa: F401,F403
from .oracle import __all__  # noqa: F401
