"""CPU oracle for the FreeSolo sparse-attention inference hot path.

TEST INFRASTRUCTURE ONLY. This package restates, in plain torch-on-CPU (fp32 arithmetic), the algorithms of the
reference's eager path so that the CUDA kernels of ``freesolo_b200`` can be checked against them. Nothing in the
product package imports it; only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` do.

Parity is pinned by execution: ``tests/golden/make_golden.py`` imports the reference itself, runs it on seeded
inputs and stores its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks every oracle function
against those stored outputs.

Each function's docstring cites the reference file:line it follows (paths relative to the reference project root).
"""
from . import fsl  # noqa: F401
