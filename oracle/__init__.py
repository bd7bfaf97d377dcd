"""CPU oracle for the einjax sparse-einsum path — TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it. Nothing under ``einjax_b200/`` imports it,
and the product path raises when its CUDA library is missing instead of
falling back here.

``einsparse_ref`` restates, in numpy, the reference's own hot-path functions
(each cites the reference ``file:line`` it follows). It is pinned against
golden vectors produced by running the unmodified reference code
(``tests/golden/make_golden.py``, committed together with its fixtures), so
parity claims rest on the reference's behaviour, not on this restatement.
"""

from .einsparse_ref import *  # noqa: F401,F403
