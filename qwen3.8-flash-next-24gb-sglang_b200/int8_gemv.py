"""INT8 dense projection GEMV for the decode step's dense linears.

In the reference these tensors run through SGLang's GPTQ Marlin INT8 kernel (third party,
docs/DECODE_PERF_PLAN.md:29); their packing is the reference's own ``pack_int8_gptq``
(scripts/requant_int8.py:32-50): uint8 values 4 per int32 along K, int32 [K/4, N], f16 scales
[K/group, N], symmetric zero point 128. ``int8_gemv`` computes y = x @ ((q - zero) * s) through the
C ABI; one scale row (``scales.shape[0] == 1``) means per-output-channel scales.
"""
from __future__ import annotations

import torch

from . import _native
from .expert_gemv import _stream

__all__ = ["int8_gemv"]

_WS8 = {}


def _ws(device, nbytes):
    key = (device.type, device.index)
    t = _WS8.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS8[key] = t
    return t


def _int8_gemv_impl(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zero: int,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    M, K = x.shape
    N = qweight.shape[1]
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device) if out is None else out
    if M == 0:
        return y
    group = K // scales.shape[0]
    nbytes = int(_native.lib().w2a16_int8_workspace_bytes(M, K, N))
    ws = _ws(x.device, nbytes)
    _native.call("w2a16_int8_gemv", x.data_ptr(), x.stride(0), qweight.data_ptr(), scales.data_ptr(), group,
                 zero, M, K, N, y.data_ptr(), y.stride(0), ws.data_ptr(), ws.numel(), _stream(x.device))
    return y


@torch.library.custom_op("w2a16_moe::int8_gemv", mutates_args=())
def _int8_gemv(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zero: int) -> torch.Tensor:
    return _int8_gemv_impl(x, qweight, scales, zero)


@_int8_gemv.register_fake
def _int8_gemv_fake(x, qweight, scales, zero):
    return x.new_empty((x.shape[0], qweight.shape[1]), dtype=torch.bfloat16)


def int8_gemv(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zero: int = 128,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """x bf16 [M, K] (or [K]), qweight int32 [K/4, N], scales f16 [K/group, N] -> bf16 [M, N]. ``out`` (bf16
    [M, N], rows contiguous, on x's device) receives the result instead of a new tensor."""
    squeeze = x.dim() == 1
    x2 = x[None] if squeeze else x
    if not (x2.is_cuda and qweight.is_cuda and scales.is_cuda):
        raise ValueError("int8_gemv needs CUDA tensors (no CPU path exists)")
    if x2.dtype != torch.bfloat16 or qweight.dtype != torch.int32 or scales.dtype != torch.float16:
        raise ValueError("int8_gemv expects x bf16, qweight int32, scales f16")
    if qweight.shape[0] * 4 != x2.shape[1]:
        raise ValueError(f"K mismatch: x {tuple(x2.shape)} vs qweight {tuple(qweight.shape)}")
    if out is not None:
        o2 = out[None] if out.dim() == 1 else out
        if o2.shape != (x2.shape[0], qweight.shape[1]) or o2.dtype != torch.bfloat16 or o2.stride(-1) != 1 \
                or o2.device != x2.device:
            raise ValueError("out must be a bf16 tensor [M, N] with contiguous rows on x's device")
        _int8_gemv_impl(x2.contiguous(), qweight.contiguous(), scales.contiguous(), int(zero), out=o2)
        return out
    op = _int8_gemv if torch.compiler.is_compiling() else _int8_gemv_impl
    y = op(x2.contiguous(), qweight.contiguous(), scales.contiguous(), int(zero))
    return y[0] if squeeze else y
