"""CPU oracle for the SunShape block-VQ KV-cache hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
module; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and
only as the checker or as the timed CPU baseline.

Parity pin: the functions here are checked against golden vectors that the
reference itself produced (``tests/golden/make_golden.py`` imports the
reference package over a NumPy-backed stand-in for ``mlx.core`` so the
reference runs its own CPU/fallback code paths) and against the explicit
NumPy known-answer computations of the reference's ``test_kernels.py``.
"""

from .sunshape_oracle import *  # noqa: F401,F403
