"""CPU oracle for the llms_b200 hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker (or the timed CPU
baseline).  The product path (``llms_b200``) never imports it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks these functions
against golden outputs produced by running the reference engine's own modules
(``tests/golden/make_golden.py``).
"""
