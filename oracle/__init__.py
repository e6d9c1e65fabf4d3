"""CPU oracle for the W2A16 g128 MoE decode path and the INT8 dense GEMV.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this package: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU baseline / ``--impl reference`` leg) may
import it, and only as the checker or as the timed CPU baseline — never as the thing measured on
the GPU or shipped. The CUDA path fails loudly when its extension is missing; it never falls back
to anything in here.

Parity pins (what this oracle is checked against, in ``tests/test_oracle_golden.py``):
  * golden vectors produced by the reference's own code (``tests/golden/make_golden.py`` imports
    ``gemv/moe_gemv_int2_tab.py`` and ``gemv/moe_gemv_int2.py`` and runs their Triton kernels under
    the Triton CPU interpreter, and executes the synthetic-data helpers of the reference's unit
    test ``test_moe_wna16_int2.py`` taken from the upstream series patch);
  * the reference's known-answer checks (bit-exact relayout and unpack, series-0002:1989-2081).
"""
from .w2moe_oracle import *  # noqa: F401,F403
