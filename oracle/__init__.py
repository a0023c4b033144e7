"""CPU oracle -- test infrastructure, never the product path.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and the
CPU-baseline leg of ``bench.py``.
"""
from .nvfp4_oracle import *  # noqa: F401,F403
