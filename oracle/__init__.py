"""CPU oracle for the W8A16 GEMM path: test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import this package, and only as the checker / the timed CPU baseline.
"""
