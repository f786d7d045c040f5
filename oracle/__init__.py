"""CPU oracle for the SSM scan hot path (TEST INFRASTRUCTURE ONLY).

Nothing in the shipped package imports this directory.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may use it,
and only as the checker or as the timed CPU baseline, never as the product path.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own
functions (imported from the reference source tree) and committed their outputs
under ``tests/golden/``; ``tests/test_oracle.py`` checks this restatement against
those fixtures.
"""

from .ssm_oracle import *  # noqa: F401,F403
