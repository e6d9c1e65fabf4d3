"""The 2-bit branch of SGLang's ``MoeWNA16Method`` as the reference patches it, on this library's kernels.

The reference adds three methods to ``MoeWNA16Method`` (patches/ncontig_gemv.py:169-255):

* ``process_weights_after_loading`` (:169-204) relayouts each layer's 2-bit expert tensors once into the
  N-contiguous word layout -- codes uint8 [E, N, K/4] -> int32 [E, K/16, N] through ``to_word_ncontig``,
  scales [E, N, K/g] -> [E, K/g, N] -- keeping offloaded (pinned host) tensors pinned, and marks the layer
  ``_b_n_contig``;
* ``_gemv_tables`` (:206-216) caches the int64 address tables of ``make_tables`` on ``layer._gemv_tabs``;
* ``apply`` (:240-255) sends a batch to the GEMV composite ``_apply_gemv`` (:218-238) when the layer is in
  the word layout, the weights are 2-bit, the batch has at most 16 tokens and ``SGLANG_MOE_GEMV`` is "1"
  (the default); every other batch goes to SGLang's tiled ``fused_experts`` (serving patch:2748-2842).

:class:`MoeWNA16Method` keeps those names, that gate and that relayout. The GEMV branch runs the whole
layer in one launch (``apply_gemv``), reading the experts wherever the tables point (device memory, or
pinned host memory for offloaded layers); the other branch is :func:`fused_experts_w2a16`, this library's
replacement of the tiled call for the word layout (the batched tensor-core path from 64 tokens, the
per-token fused layer below). Optional per-group 2-bit zero points (``w13_qzeros`` / ``w2_qzeros`` in the
loader form [E, N/4, K/g]) are relayouted to the GEMV form and used by both branches.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from .expert_gemv import make_tables, make_zero_table, to_word_ncontig, zeros_to_ncontig
from .moe_layer import ExpertArena, apply_gemv, moe_decode_layer

__all__ = ["GEMV_MAX_TOKENS", "use_gemv", "MoeWNA16Method", "fused_experts_w2a16"]

GEMV_MAX_TOKENS = 16          # the apply gate's batch limit (patches/ncontig_gemv.py:252)

_NAMES = ("w13_qweight", "w2_qweight", "w13_scales", "w2_scales")


def use_gemv(layer, num_tokens: int, weight_bits: int = 2, env=None) -> bool:
    """The reference's gate (patches/ncontig_gemv.py:249-253): word layout, 2-bit, at most 16 tokens and
    ``SGLANG_MOE_GEMV`` unset or "1"."""
    env = os.environ if env is None else env
    return (bool(getattr(layer, "_b_n_contig", False)) and weight_bits == 2
            and num_tokens <= GEMV_MAX_TOKENS and env.get("SGLANG_MOE_GEMV", "1") == "1")


def _data(t):
    return t.data if isinstance(t, torch.nn.Parameter) else t


def _set(layer, name, value):
    p = getattr(layer, name)
    if isinstance(p, torch.nn.Parameter):
        p.data = value
    else:
        setattr(layer, name, value)


def fused_experts_w2a16(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                        topk_weights: torch.Tensor, topk_ids: torch.Tensor, w1_scale: torch.Tensor,
                        w2_scale: torch.Tensor, w1_zp: Optional[torch.Tensor] = None,
                        w2_zp: Optional[torch.Tensor] = None,
                        routed_scaling_factor: Optional[float] = None) -> torch.Tensor:
    """The tiled ``fused_experts`` call for 2-bit experts in the word layout (serving patch:2748-2842 with
    ``use_int2_w2a16``; its kernel ``fused_moe_kernel_gptq_awq_word``, serving patch:9-295): w1 int32
    [E, H/16, 2I] (gate rows [0, I), up [I, 2I)), w2 int32 [E, I/16, H], scales [E, K/128, N], zero points
    uint8 [E, K/128, N/4] (GEMV form) or None for the symmetric zero point 2. hidden_states bf16 [M, H],
    topk_ids / topk_weights [M, top_k] -> bf16 [M, H] = routed_scaling_factor * sum_j w_j * down(silu(gate)
    * up). The experts are used in place as an arena with the identity slot table; from 64 tokens the
    library takes its batched path (each routed expert streamed once, tcgen05 MMAs), below it the per-token
    fused layer. Device tensors only (an offloaded layer's small batches go through the GEMV branch)."""
    arena = ExpertArena(w1, w1_scale, w2, w2_scale, w1_zp, w2_zp)
    rsf = 1.0 if routed_scaling_factor is None else float(routed_scaling_factor)
    return moe_decode_layer(hidden_states, topk_ids, topk_weights, arena, rsf)


class MoeWNA16Method:
    """The reference's 2-bit ``MoeWNA16Method`` paths over a layer object holding ``w13_qweight``,
    ``w2_qweight``, ``w13_scales``, ``w2_scales`` (tensors or Parameters) and optionally ``w13_qzeros`` /
    ``w2_qzeros``."""

    def __init__(self, weight_bits: int = 2, routed_scaling_factor: Optional[float] = None):
        self.weight_bits = int(weight_bits)
        self.routed_scaling_factor = routed_scaling_factor

    def process_weights_after_loading(self, layer) -> None:
        """Relayout once into the word layout (patches/ncontig_gemv.py:169-204): codes through
        ``to_word_ncontig``, scales transposed to [E, K/g, N]; pinned host tensors stay pinned. The
        ``SGLANG_MOE_NCONTIG`` switch ("1" by default) is honoured; zero points, when present, go to the
        GEMV form [E, K/g, N/4]."""
        if self.weight_bits != 2 or os.environ.get("SGLANG_MOE_NCONTIG", "1") != "1":
            return
        for name in _NAMES:
            p = getattr(layer, name, None)
            t = None if p is None else _data(p)
            if t is None or t.dim() != 3:
                continue
            was_pinned = (not t.is_cuda) and t.is_pinned()
            t2 = to_word_ncontig(t) if name.endswith("qweight") else t.transpose(1, 2).contiguous()
            if was_pinned and not t2.is_pinned():
                t2 = t2.pin_memory()
            _set(layer, name, t2)
        for name in ("w13_qzeros", "w2_qzeros"):
            z = getattr(layer, name, None)
            if z is not None:
                z2 = zeros_to_ncontig(_data(z))
                if (not z2.is_cuda) and _data(z).is_pinned() and not z2.is_pinned():
                    z2 = z2.pin_memory()
                _set(layer, name, z2)
        layer._b_n_contig = True
        layer._gemv_tabs = None

    def _gemv_tables(self, layer):
        """The cached table tuple of patches/ncontig_gemv.py:206-216 (``layer._gemv_tabs = None``
        invalidates it)."""
        tabs = getattr(layer, "_gemv_tabs", None)
        if tabs is None:
            w13, s13 = _data(layer.w13_qweight), _data(layer.w13_scales)
            w2, s2 = _data(layer.w2_qweight), _data(layer.w2_scales)
            tabs = (make_tables(w13, s13), make_tables(w2, s2), w13.shape[2], w13.shape[1] * 16,
                    w2.shape[2], w2.shape[1] * 16, s13.dtype == torch.bfloat16)
            layer._gemv_tabs = tabs
            z13, z2 = getattr(layer, "w13_qzeros", None), getattr(layer, "w2_qzeros", None)
            layer._gemv_zero_tabs = None if z13 is None else (make_zero_table(_data(z13))[0],
                                                              make_zero_table(_data(z2))[0])
        return tabs

    def _apply_gemv(self, layer, hidden_states, topk_ids, topk_weights) -> torch.Tensor:
        """The batch-1 composite (patches/ncontig_gemv.py:218-238) as one fused launch."""
        tabs = self._gemv_tables(layer)
        return apply_gemv(hidden_states, topk_ids, topk_weights, tabs, self.routed_scaling_factor,
                          zero_tabs=getattr(layer, "_gemv_zero_tabs", None)).to(hidden_states.dtype)

    def apply(self, layer, hidden_states: torch.Tensor, topk_ids: torch.Tensor,
              topk_weights: torch.Tensor) -> torch.Tensor:
        """The reference's dispatch (patches/ncontig_gemv.py:240-255): the GEMV composite for small
        batches on word-layout 2-bit layers, else the tiled path (:func:`fused_experts_w2a16`)."""
        if use_gemv(layer, hidden_states.shape[0], self.weight_bits):
            return self._apply_gemv(layer, hidden_states, topk_ids, topk_weights)
        z13, z2 = getattr(layer, "w13_qzeros", None), getattr(layer, "w2_qzeros", None)
        return fused_experts_w2a16(hidden_states, _data(layer.w13_qweight), _data(layer.w2_qweight), topk_weights,
                                   topk_ids, _data(layer.w13_scales), _data(layer.w2_scales),
                                   None if z13 is None else _data(z13), None if z2 is None else _data(z2),
                                   self.routed_scaling_factor)
