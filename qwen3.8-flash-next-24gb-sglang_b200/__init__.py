"""B200-native (sm_100a) W2A16 group-128 MoE decode GEMV — drop-in for the reference's expert GEMV path.

Public API (mirrors the reference's ``expert_gemv`` module and ``MoeWNA16Method._apply_gemv``):

* :func:`moe_gemv_int2_tab`, :func:`make_tables`, :func:`to_word_ncontig` — the reference's three
  names with their signatures (gemv/moe_gemv_int2_tab.py:72-109);
* :func:`moe_decode_layer` / :func:`apply_gemv` — the whole decode MoE layer in one call
  (patches/ncontig_gemv.py:218-238), over an int32 slot table (:class:`ExpertArena`) or the
  reference's int64 address tables;
* :class:`MoeWNA16Method` / :func:`use_gemv` / :func:`fused_experts_w2a16` — the caller's 2-bit
  dispatch (patches/ncontig_gemv.py:169-255): load-time relayout, the M <= 16 / ``SGLANG_MOE_GEMV`` gate,
  and the tiled branch for larger batches;
* :mod:`arena` — native expert arenas (reserved virtual addresses, chunks mapped on growth and released on
  shrink; an elastic layer arena with an in-place slot table), the reference's ``RowArena`` / elastic resize;
* :func:`int8_gemv` — the INT8 dense projection GEMV;
* :mod:`expert_parallel` — experts split across GPUs (one process per GPU, NCCL all-reduce).

All compute runs in ``lib/libw2a16_moe.so`` (hand-written CUDA for sm_100a) behind the C ABI of
``include/w2a16_moe.h``; there is no CPU fallback.
"""
from ._native import lib, version, W2A16Error  # noqa: F401
from .expert_gemv import (moe_gemv_int2_tab, make_tables, make_zero_table, to_word_ncontig,  # noqa: F401
                          zeros_to_ncontig, moe_gemv_int2_slots, last_device_error)
from .moe_layer import ExpertArena, moe_decode_layer, apply_gemv  # noqa: F401
from .moe_method import MoeWNA16Method, use_gemv, fused_experts_w2a16  # noqa: F401
from .int8_gemv import int8_gemv  # noqa: F401
from . import synth  # noqa: F401
from . import expert_parallel  # noqa: F401
from . import arena  # noqa: F401
