"""Drop-in for the reference's ``expert_gemv`` module.

The reference ships ``gemv/moe_gemv_int2_tab.py`` and installs it into SGLang as
``sglang/srt/layers/moe/expert_gemv.py`` (patches/ncontig_gemv.py:25-26, :324); its callers are
``MoeWNA16Method._apply_gemv`` / ``_gemv_tables`` / ``process_weights_after_loading``
(patches/ncontig_gemv.py:169-238) and the placement patch (patches/placement.py:208-227). This
module keeps the three public names and their call signatures:

    moe_gemv_int2_tab(a, wtab, stab, topk_ids, topk_w, N, K, stride_ww, stride_sg, top_k,
                      mul_routed_weight, block_n=64, block_k=128, num_warps=4, scale_bf16=True)
    make_tables(qweight, scales) -> (wtab, stab, stride_ww, stride_sg)
    to_word_ncontig(qweight_u8_nk) -> int32 [E, K/16, N]

and adds optional keyword arguments only (``ztab``/``stride_zg`` for per-group 2-bit zero points).
Every call goes through a torch custom op into the C ABI of ``lib/libw2a16_moe.so``; there is no
Triton and no CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _native

__all__ = ["moe_gemv_int2_tab", "make_tables", "make_zero_table", "to_word_ncontig", "zeros_to_ncontig",
           "moe_gemv_int2_slots", "last_device_error"]

_ERR = {}


def _err_word(device: torch.device) -> torch.Tensor:
    """Per-device uint32 error word the kernels OR their error bits into."""
    key = (device.type, device.index)
    t = _ERR.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[key] = t
    return t


def last_device_error(device=None, reset: bool = True) -> int:
    """Read (and by default clear) the device error bits: 1 = expert id out of range, 2 = a bounded
    wait gave up. Synchronises with the device; meant for tests and debugging, not the hot path."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    t = _err_word(dev)
    v = int(t.item())
    if reset:
        t.zero_()
    return v


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


@torch.library.custom_op("w2a16_moe::gemv_tab", mutates_args=())
def _gemv_tab(a: torch.Tensor, wtab: torch.Tensor, stab: torch.Tensor, ztab: Optional[torch.Tensor],
              topk_ids: torch.Tensor, topk_w: Optional[torch.Tensor], N: int, K: int, stride_ww: int,
              stride_sg: int, stride_zg: int, top_k: int, mul_routed_weight: bool,
              scale_bf16: bool) -> torch.Tensor:
    R = topk_ids.numel()
    c = torch.empty((R, N), dtype=torch.bfloat16, device=a.device)
    if R == 0:
        return c
    _native.call("w2a16_moe_gemv_tab", a.data_ptr(), a.stride(0), wtab.data_ptr(), stab.data_ptr(), _p(ztab),
                 wtab.numel(), topk_ids.data_ptr(), _p(topk_w), c.data_ptr(), c.stride(0), R, N, K,
                 stride_ww, stride_sg, stride_zg, top_k, int(mul_routed_weight), int(scale_bf16),
                 _err_word(a.device).data_ptr(), _stream(a.device))
    return c


@_gemv_tab.register_fake
def _gemv_tab_fake(a, wtab, stab, ztab, topk_ids, topk_w, N, K, stride_ww, stride_sg, stride_zg, top_k,
                   mul_routed_weight, scale_bf16):
    return a.new_empty((topk_ids.numel(), N), dtype=torch.bfloat16)


def _check_cuda(name: str, t: torch.Tensor, dtype=None):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path exists), got {t.device}")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")


def moe_gemv_int2_tab(a, wtab, stab, topk_ids, topk_w, N, K, stride_ww, stride_sg, top_k,
                      mul_routed_weight, block_n=64, block_k=128, num_warps=4, scale_bf16=True,
                      ztab=None, stride_zg=None):
    """a [M, K] bf16; topk_ids/topk_w flat [R]; returns bf16 [R, N] (gemv/moe_gemv_int2_tab.py:72-85).

    Row r uses expert topk_ids[r] and activation row r // top_k; with ``mul_routed_weight`` the row is
    scaled by topk_w[r]. ``block_n``/``num_warps`` are accepted for signature compatibility (the CUDA
    kernel's tiling is fixed); ``block_k`` keeps the reference's check. ``ztab`` (int64 [E] addresses of
    uint8 [K/128, N/4] zero-point rows) switches from the symmetric zero point 2 to per-group zeros."""
    assert K % block_k == 0 and block_k % 128 == 0, (K, block_k)   # the reference's own check (:77)
    _check_cuda("a", a, torch.bfloat16)
    _check_cuda("topk_ids", topk_ids)
    if a.stride(-1) != 1:
        a = a.contiguous()
    ids = topk_ids.reshape(-1)
    if ids.dtype != torch.int32:
        ids = ids.to(torch.int32)
    ids = ids.contiguous()
    w = None
    if mul_routed_weight:
        w = topk_w.reshape(-1).to(torch.float32).contiguous()
    elif topk_w is not None:
        w = topk_w.reshape(-1).to(torch.float32).contiguous()
    zg = int(stride_zg) if stride_zg is not None else (N // 4)
    return _gemv_tab(a, wtab, stab, ztab, ids, w, int(N), int(K), int(stride_ww), int(stride_sg), zg,
                     int(top_k), bool(mul_routed_weight), bool(scale_bf16))


def make_tables(qweight: torch.Tensor, scales: torch.Tensor):
    """qweight int32 [E, K/16, N], scales f16/bf16 [E, K/128, N] (contiguous) -> int64 [E] address
    tables on the CUDA device plus the row strides in elements (gemv/moe_gemv_int2_tab.py:88-97)."""
    assert qweight.dtype == torch.int32 and scales.dtype in (torch.float16, torch.bfloat16), \
        (qweight.dtype, scales.dtype)
    assert qweight.is_contiguous() and scales.is_contiguous()
    E = qweight.shape[0]
    dev = qweight.device if qweight.is_cuda else torch.device("cuda")
    wt = torch.arange(E, dtype=torch.int64) * (qweight.stride(0) * 4) + qweight.data_ptr()
    st = torch.arange(E, dtype=torch.int64) * (scales.stride(0) * scales.element_size()) + scales.data_ptr()
    return wt.to(dev), st.to(dev), qweight.stride(1), scales.stride(1)


def make_zero_table(zeros: torch.Tensor):
    """zeros uint8 [E, K/128, N/4] (GEMV form, see :func:`zeros_to_ncontig`) -> (int64 [E] addresses
    on the CUDA device, bytes per group row)."""
    assert zeros.dtype == torch.uint8 and zeros.is_contiguous() and zeros.dim() == 3
    E = zeros.shape[0]
    dev = zeros.device if zeros.is_cuda else torch.device("cuda")
    zt = torch.arange(E, dtype=torch.int64) * zeros.stride(0) + zeros.data_ptr()
    return zt.to(dev), zeros.stride(1)


@torch.library.custom_op("w2a16_moe::to_word_ncontig", mutates_args=())
def _to_word(src: torch.Tensor) -> torch.Tensor:
    E, N, KB = src.shape
    out = torch.empty((E, KB // 4, N), dtype=torch.int32, device=src.device)
    _native.call("w2a16_to_word_ncontig", src.data_ptr(), out.data_ptr(), E, N, KB * 4, _stream(src.device))
    return out


@_to_word.register_fake
def _to_word_fake(src):
    E, N, KB = src.shape
    return src.new_empty((E, KB // 4, N), dtype=torch.int32)


def _to_word_host(src: torch.Tensor) -> torch.Tensor:
    """The relayout of a host tensor, run by the same CUDA kernel: the GPU reads the pinned source and writes a
    pinned result through unified addressing (no CPU arithmetic). A pageable source is first copied into
    pinned memory. Synchronises the stream before returning, as the host result is used right away."""
    if not torch.cuda.is_available():
        raise RuntimeError("to_word_ncontig of a host tensor runs on the GPU through unified addressing; "
                           "no CUDA device is available (there is no CPU path)")
    E, N, KB = src.shape
    pinned = src if src.is_pinned() else src.pin_memory()
    out = torch.empty((E, KB // 4, N), dtype=torch.int32).pin_memory()
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    _native.call("w2a16_to_word_ncontig", pinned.data_ptr(), out.data_ptr(), E, N, KB * 4, stream.cuda_stream)
    stream.synchronize()
    return out


def to_word_ncontig(qweight_u8_nk: torch.Tensor) -> torch.Tensor:
    """Loader layout uint8 [E, N, K/4] -> int32 [E, K/16, N], bit-exact (gemv/moe_gemv_int2_tab.py:100-109):
    byte kb of row n becomes byte kb % 4 of word kb // 4 at column n. Runs as a CUDA kernel. A CUDA tensor
    gives a CUDA tensor (asynchronous, current stream); a host tensor -- the reference relayouts offloaded
    experts that live in pinned host memory (patches/ncontig_gemv.py:195-201) -- gives a pinned host tensor,
    the kernel reading and writing host memory over the bus (the call waits for it)."""
    if qweight_u8_nk.dtype != torch.uint8:
        raise ValueError(f"qweight_u8_nk must be uint8, got {qweight_u8_nk.dtype}")
    assert qweight_u8_nk.dim() == 3 and qweight_u8_nk.shape[2] % 4 == 0, qweight_u8_nk.shape
    if not qweight_u8_nk.is_cuda:
        return _to_word_host(qweight_u8_nk.contiguous())
    return _to_word(qweight_u8_nk.contiguous())


def zeros_to_ncontig(qzeros: torch.Tensor) -> torch.Tensor:
    """Loader form uint8 [E, N/4, K/g] (series-0002:1946-1947) -> GEMV form uint8 [E, K/g, N/4]."""
    assert qzeros.dtype == torch.uint8 and qzeros.dim() == 3
    return qzeros.transpose(1, 2).contiguous()


@torch.library.custom_op("w2a16_moe::gemv_slots", mutates_args=())
def _gemv_slots(a: torch.Tensor, slots: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor,
                zeros: Optional[torch.Tensor], topk_ids: torch.Tensor, topk_w: Optional[torch.Tensor],
                top_k: int, mul_routed_weight: bool) -> torch.Tensor:
    R = topk_ids.numel()
    N = codes.shape[2]
    K = codes.shape[1] * 16
    c = torch.empty((R, N), dtype=torch.bfloat16, device=a.device)
    if R == 0:
        return c
    _native.call("w2a16_moe_gemv_slots", a.data_ptr(), a.stride(0), slots.data_ptr(), slots.numel(), codes.shape[0],
                 codes.data_ptr(), codes.stride(0) * 4, scales.data_ptr(), scales.stride(0) * scales.element_size(),
                 _p(zeros), 0 if zeros is None else zeros.stride(0), topk_ids.data_ptr(), _p(topk_w),
                 c.data_ptr(), c.stride(0), R, N, K, top_k, int(mul_routed_weight),
                 int(scales.dtype == torch.bfloat16), _err_word(a.device).data_ptr(), _stream(a.device))
    return c


@_gemv_slots.register_fake
def _gemv_slots_fake(a, slots, codes, scales, zeros, topk_ids, topk_w, top_k, mul_routed_weight):
    return a.new_empty((topk_ids.numel(), codes.shape[2]), dtype=torch.bfloat16)


def moe_gemv_int2_slots(a, slots, codes, scales, topk_ids, topk_w=None, top_k=1, mul_routed_weight=False,
                        zeros=None):
    """The GEMV over an expert arena: codes int32 [S, K/16, N], scales [S, K/128, N], zeros uint8
    [S, K/128, N/4] or None, slots int32 [E] (slot -1 = not resident -> zero row). Returns bf16 [R, N]."""
    _check_cuda("a", a, torch.bfloat16)
    _check_cuda("slots", slots, torch.int32)
    _check_cuda("codes", codes, torch.int32)
    assert codes.is_contiguous() and scales.is_contiguous() and (zeros is None or zeros.is_contiguous())
    ids = topk_ids.reshape(-1).to(torch.int32).contiguous()
    w = None if topk_w is None else topk_w.reshape(-1).to(torch.float32).contiguous()
    if mul_routed_weight and w is None:
        raise ValueError("mul_routed_weight needs topk_w")
    return _gemv_slots(a.contiguous(), slots.contiguous(), codes, scales, zeros, ids, w, int(top_k),
                       bool(mul_routed_weight))
