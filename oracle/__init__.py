"""Test infrastructure only: CPU restatements of the reference RACE attention path.

Nothing in the product package imports this directory.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arms use
it, and only as the checker or as the timed CPU baseline.
"""
