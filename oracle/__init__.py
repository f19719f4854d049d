"""CPU oracle for the Neso B200 kernels — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg (and its ``--impl reference`` arm) may import this package, and only as the
checker or the timed CPU baseline. The product path (``neso_b200``) never
imports it and has no CPU fallback.
"""
from .oracle import *  # noqa: F401,F403
