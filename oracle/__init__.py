"""CPU oracle for the MoE decode hot path: TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this package, and only as the checker or the timed CPU
baseline.  The product path (``wanferenz_b200``) never imports it.
"""
