"""Test-only oracle: a CPU fp32 restatement of the reference forward.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker.
"""
