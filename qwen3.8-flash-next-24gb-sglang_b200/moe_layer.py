"""Decode MoE layer: gate_up GEMV + SiLU*mul + down GEMV * routed weight + top-k sum.

Replaces ``MoeWNA16Method._apply_gemv`` (patches/ncontig_gemv.py:218-238), which runs two
``moe_gemv_int2_tab`` launches with torch SiLU*mul and a torch top-k sum in between, by one C-ABI
call. Two addressing forms:

* :func:`apply_gemv` takes the reference's cached table tuple (``_gemv_tables``,
  patches/ncontig_gemv.py:206-216 / patches/placement.py:208-227): int64 address tables per expert;
* :func:`moe_decode_layer` takes an :class:`ExpertArena`: stacked expert tensors indexed through an
  int32 slot table, slot -1 = expert not resident (its routed rows contribute zero).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import _native
from .expert_gemv import _err_word, _p, _stream

__all__ = ["ExpertArena", "moe_decode_layer", "apply_gemv", "layer_workspace"]

_WS = {}


def layer_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device workspace (uint8, zero-filled on creation, grown on demand). The layer kernels leave
    its control words consistent after every call (barrier count equal to its generation, hand-off words
    tagged with past calls' epochs), so it is reused without clearing."""
    key = (device.type, device.index)
    t = _WS.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = t
    return t


@dataclass
class ExpertArena:
    """One MoE layer's experts in arena form.

    codes13 int32 [S, H/16, 2I]   gate rows [0, I), up rows [I, 2I)  (gemv/test_gemv_tab.py:32)
    scales13 f16|bf16 [S, H/128, 2I]
    codes2  int32 [S, I/16, H]
    scales2 f16|bf16 [S, I/128, H]
    zeros13 / zeros2 uint8 [S, K/128, N/4] or None (symmetric zero point 2)
    slots   int32 [E]: slot of expert e, -1 = not resident. ``None`` = identity (S == E).
    """
    codes13: torch.Tensor
    scales13: torch.Tensor
    codes2: torch.Tensor
    scales2: torch.Tensor
    zeros13: Optional[torch.Tensor] = None
    zeros2: Optional[torch.Tensor] = None
    slots: Optional[torch.Tensor] = None

    def __post_init__(self):
        for n in ("codes13", "scales13", "codes2", "scales2"):
            t = getattr(self, n)
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{n} must be a contiguous CUDA tensor")
        if self.codes13.dtype != torch.int32 or self.codes2.dtype != torch.int32:
            raise ValueError("codes must be int32 words")
        if self.scales13.dtype != self.scales2.dtype or self.scales13.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("scales must be f16 or bf16 (both tensors the same)")
        if (self.zeros13 is None) != (self.zeros2 is None):
            raise ValueError("zeros13 and zeros2 must both be given or both be None")
        S = self.codes13.shape[0]
        for n in ("scales13", "codes2", "scales2", "zeros13", "zeros2"):
            t = getattr(self, n)
            if t is not None and t.shape[0] != S:
                raise ValueError(f"{n} holds {t.shape[0]} slots, codes13 {S}: every arena tensor needs the same slots")
        if self.slots is None:
            self.slots = torch.arange(S, dtype=torch.int32, device=self.codes13.device)
        if self.slots.dtype != torch.int32 or not self.slots.is_cuda:
            raise ValueError("slots must be an int32 CUDA tensor")

    @property
    def H(self) -> int:
        return self.codes13.shape[1] * 16

    @property
    def I(self) -> int:  # noqa: E743
        return self.codes13.shape[2] // 2

    @property
    def E(self) -> int:
        return self.slots.numel()

    @property
    def S(self) -> int:
        return self.codes13.shape[0]

    @property
    def scale_bf16(self) -> bool:
        return self.scales13.dtype == torch.bfloat16

    def bytes_per_expert(self) -> int:
        """Algorithmic bytes one routed expert streams (codes + scales + zeros of gate_up and down)."""
        n = 0
        for t in (self.codes13, self.scales13, self.codes2, self.scales2, self.zeros13, self.zeros2):
            if t is not None:
                n += t[0].numel() * t.element_size()
        return n


_WS_BYTES = {}


BATCHED_MIN_TOKENS = _native.BATCHED_AUTO_TOKENS   # the library's own choice: the batched path from here
BATCHED_FORCE_MIN_TOKENS = 16                      # the batched path's smallest token count


def _path(M: int, batched: int) -> int:
    """C-ABI path choice for a slot-form call. batched -1: the library's choice by token count (the batched
    path from BATCHED_MIN_TOKENS tokens, where it is the faster one); 1: the batched path from 16 tokens (the
    per-token path below); 0: the per-token path."""
    if batched == 0 or (batched == 1 and M < BATCHED_FORCE_MIN_TOKENS):
        return _native.PATH_PER_TOKEN
    return _native.PATH_BATCHED if batched == 1 else _native.PATH_AUTO


def _workspace_bytes(M: int, H: int, I: int, top_k: int, batched: int = -1) -> int:
    """Workspace bytes of a slot-form layer call taking the path _path(M, batched) chooses: the batched path's
    size where that path runs, else the per-token path's."""
    key = (M, H, I, top_k, batched)
    n = _WS_BYTES.get(key)
    if n is None:
        lib = _native.lib()
        path = _path(M, batched)
        if path == _native.PATH_BATCHED or (path == _native.PATH_AUTO and M >= BATCHED_MIN_TOKENS):
            n = int(lib.w2a16_moe_layer_workspace_bytes_batched(M, H, I, top_k))
        else:
            n = int(lib.w2a16_moe_layer_workspace_bytes(M, H, I, top_k))
        _WS_BYTES[key] = n
    return n


def _decode_layer_slots_impl(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, slots: torch.Tensor,
                             codes13: torch.Tensor, scales13: torch.Tensor, zeros13: Optional[torch.Tensor],
                             codes2: torch.Tensor, scales2: torch.Tensor, zeros2: Optional[torch.Tensor],
                             routed_scaling_factor: float, batched: int = -1,
                             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    M, H = x.shape
    top_k = topk_ids.shape[1]
    I = codes13.shape[2] // 2
    y = torch.empty((M, H), dtype=torch.bfloat16, device=x.device) if out is None else out
    if M == 0:
        return y
    nbytes = _workspace_bytes(M, H, I, top_k, batched)
    ws = layer_workspace(x.device, nbytes)
    esz = scales13.element_size()
    _native.call("w2a16_moe_decode_layer_slots_ex", x.data_ptr(), M, H, I, top_k, topk_ids.data_ptr(),
                 topk_w.data_ptr(), slots.data_ptr(), slots.numel(), codes13.shape[0],
                 codes13.data_ptr(), codes13.stride(0) * 4, scales13.data_ptr(), scales13.stride(0) * esz,
                 _p(zeros13), 0 if zeros13 is None else zeros13.stride(0),
                 codes2.data_ptr(), codes2.stride(0) * 4, scales2.data_ptr(), scales2.stride(0) * esz,
                 _p(zeros2), 0 if zeros2 is None else zeros2.stride(0),
                 int(scales13.dtype == torch.bfloat16), float(routed_scaling_factor), y.data_ptr(),
                 ws.data_ptr(), nbytes, _path(M, batched), _err_word(x.device).data_ptr(), _stream(x.device))
    return y


@torch.library.custom_op("w2a16_moe::decode_layer_slots", mutates_args=())
def _decode_layer_slots(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, slots: torch.Tensor,
                        codes13: torch.Tensor, scales13: torch.Tensor, zeros13: Optional[torch.Tensor],
                        codes2: torch.Tensor, scales2: torch.Tensor, zeros2: Optional[torch.Tensor],
                        routed_scaling_factor: float, batched: int = -1) -> torch.Tensor:
    return _decode_layer_slots_impl(x, topk_ids, topk_w, slots, codes13, scales13, zeros13, codes2, scales2,
                                    zeros2, routed_scaling_factor, batched)


@_decode_layer_slots.register_fake
def _decode_layer_slots_fake(x, topk_ids, topk_w, slots, codes13, scales13, zeros13, codes2, scales2, zeros2,
                             routed_scaling_factor, batched=-1):
    return torch.empty_like(x, dtype=torch.bfloat16)


def _routing(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor):
    if not x.is_cuda or x.dtype != torch.bfloat16:
        raise ValueError("x must be a bf16 CUDA tensor (no CPU path exists)")
    if topk_ids.dim() != 2 or topk_ids.shape[0] != x.shape[0]:
        raise ValueError(f"topk_ids must be [M, top_k], got {tuple(topk_ids.shape)}")
    ids = topk_ids.to(torch.int32).contiguous()
    w = topk_weights.to(torch.float32).contiguous()
    return x.contiguous(), ids, w


def moe_decode_layer(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, arena: ExpertArena,
                     routed_scaling_factor: float = 1.0, batched: Optional[bool] = None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[m] = routed_scaling_factor * sum_j w[m, j] * down_e(silu(gate_e(x_m)) * up_e(x_m)),
    e = topk_ids[m, j] looked up through ``arena.slots``. x bf16 [M, H] -> bf16 [M, H].

    ``batched``: None lets the library choose (the batched path -- routed rows grouped by expert, each
    expert streamed once, products on the tensor cores -- from 64 tokens, where it is faster than the
    per-token path); True takes it from 16 tokens; False always takes the per-token path. ``out`` (bf16
    [M, H], contiguous, on x's device) receives the result instead of a new tensor -- a decode loop that
    chains layers through fixed buffers then runs no copy kernel between them."""
    x, ids, w = _routing(x, topk_ids, topk_weights)
    b = -1 if batched is None else int(bool(batched))
    args = (x, ids, w, arena.slots, arena.codes13, arena.scales13, arena.zeros13, arena.codes2, arena.scales2,
            arena.zeros2, float(routed_scaling_factor), b)
    if torch.compiler.is_compiling():
        # traced/compiled code goes through the registered op (functional: the result is copied into out)
        y = _decode_layer_slots(*args)
        return y if out is None else out.copy_(y)
    if out is not None and (out.shape != x.shape or out.dtype != torch.bfloat16 or not out.is_contiguous()
                            or out.device != x.device):
        raise ValueError("out must be a contiguous bf16 tensor shaped like x on x's device")
    # eager calls skip the custom-op dispatcher (tens of microseconds of host time)
    return _decode_layer_slots_impl(*args, out=out)


@torch.library.custom_op("w2a16_moe::decode_layer_tab", mutates_args=())
def _decode_layer_tab(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, wtab13: torch.Tensor,
                      stab13: torch.Tensor, ztab13: Optional[torch.Tensor], wtab2: torch.Tensor,
                      stab2: torch.Tensor, ztab2: Optional[torch.Tensor], I: int, scale_bf16: bool,
                      routed_scaling_factor: float) -> torch.Tensor:
    M, H = x.shape
    top_k = topk_ids.shape[1]
    y = torch.empty((M, H), dtype=torch.bfloat16, device=x.device)
    if M == 0:
        return y
    nbytes = int(_native.lib().w2a16_moe_layer_workspace_bytes(M, H, I, top_k))
    ws = layer_workspace(x.device, nbytes)
    _native.call("w2a16_moe_decode_layer_tab", x.data_ptr(), M, H, I, top_k, topk_ids.data_ptr(),
                 topk_w.data_ptr(), wtab13.numel(), wtab13.data_ptr(), stab13.data_ptr(), _p(ztab13),
                 wtab2.data_ptr(), stab2.data_ptr(), _p(ztab2), int(scale_bf16), float(routed_scaling_factor),
                 y.data_ptr(), ws.data_ptr(), ws.numel(), _err_word(x.device).data_ptr(), _stream(x.device))
    return y


@_decode_layer_tab.register_fake
def _decode_layer_tab_fake(x, topk_ids, topk_w, wtab13, stab13, ztab13, wtab2, stab2, ztab2, I, scale_bf16,
                           routed_scaling_factor):
    return torch.empty_like(x, dtype=torch.bfloat16)


def apply_gemv(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, tabs,
               routed_scaling_factor: Optional[float] = None, zero_tabs=None) -> torch.Tensor:
    """The reference's ``_apply_gemv`` on its cached tables (patches/ncontig_gemv.py:218-238).

    ``tabs`` = ((wt13, st13, sw13, ss13), (wt2, st2, sw2, ss2), N13, K13, N2, K2, scale_bf16) as built by
    ``_gemv_tables`` (:206-216). The strides must be the dense ones (sw13 == ss13 == N13,
    sw2 == ss2 == N2). ``zero_tabs`` = (zt13, zt2) int64 address tables of per-group zero points or None.
    Returns the combined hidden states [M, H] in x's dtype (bf16)."""
    (wt13, st13, sw13, ss13), (wt2, st2, sw2, ss2), N13, K13, N2, K2, sbf = tabs
    if sw13 != N13 or ss13 != N13 or sw2 != N2 or ss2 != N2:
        raise ValueError("apply_gemv expects dense expert tensors (row strides equal to N)")
    if K2 * 2 != N13 or N2 != K13:
        raise ValueError(f"inconsistent layer shapes N13={N13} K13={K13} N2={N2} K2={K2}")
    x, ids, w = _routing(x, topk_ids, topk_weights)
    zt13, zt2 = (None, None) if zero_tabs is None else zero_tabs
    rsf = 1.0 if routed_scaling_factor is None else float(routed_scaling_factor)
    return _decode_layer_tab(x, ids, w, wt13, st13, zt13, wt2, st2, zt2, N13 // 2, bool(sbf), rsf)
