"""CPU oracle for the pax_b200 GEMM path.

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg of ``bench.py`` may import this package, and only as the
checker or as the timed CPU baseline.  The library under test never imports
it and has no CPU fallback.
"""
from .oracle import *  # noqa: F401,F403
