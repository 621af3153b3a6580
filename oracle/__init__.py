"""Test infrastructure: CPU restatement of the reference's VC-Attention hot path.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` import this package, as the checker or the timed CPU baseline.
The product package never does.
"""
