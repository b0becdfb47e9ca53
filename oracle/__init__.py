"""CPU oracle for the SparsePR attention hot path (test infrastructure only).

This package restates, in plain PyTorch on the CPU, the algorithm that the
reference SparsePR implementation (``src/sparsepr``) runs for one
``--attention sparsepr`` call.  Every function cites the reference file and
line range it follows.  It exists to CHECK the CUDA product path: only the
tests, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import it.  Nothing in ``sparsepr_b200``
imports this package.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own CPU code
(``N8V6Core.route``/``repair`` with the reference's torch k-means fallback and
torch gather permute) on config-0 inputs and records the outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle against
those vectors and against the reference's only known-answer test (the selector
example in ``tests/test_n8_extension.py:79-103``).
"""

from .n8_oracle import *  # noqa: F401,F403
