"""CPU checkers for the Weaver decode attention — TEST INFRASTRUCTURE ONLY.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py``; see ``oracle/checker.py``.
"""
from .checker import *  # noqa: F401,F403
from .checker import (ORACLE_SO, REF_SO, SPARSE_CODE_DTYPE, block_entropy, build, config_decode,  # noqa: F401
                      distill_rows, f2h, h2f, literal_decode, ref_available)
