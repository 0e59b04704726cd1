"""CPU oracle (test infrastructure only; see ``oracle/ops.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker or the timed CPU baseline.
"""
