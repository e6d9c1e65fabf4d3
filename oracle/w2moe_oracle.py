"""CPU restatement of the reference's W2A16 g128 MoE decode math and its INT8 dense projection.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Every function is a plain torch-on-CPU
restatement of the reference's own torch formulation, written for this repository; each docstring
names the reference lines it follows (paths relative to the reference checkout; "series-0002" is
``sglang/upstream/series-base/0002-feat-moe_wna16-2-bit-experts-expert-streaming-N-cont.patch``,
"serving patch" is ``sglang/qwen4exp-serving-73a255206f.patch``).

Layouts (shared with the CUDA path):
  codes   int32 [E, K/16, N]   value k of column n at bits 2*(k%16) of word k//16, N contiguous
  scales  f16|bf16 [E, K/128, N]
  zeros   uint8 [E, K/128, N/4] (N-contiguous form used by the GEMV; zero point of column n at bits
          2*(n%4) of byte n//4). The reference's loader form is uint8 [E, N/4, K/128]
          (series-0002:1946-1947); ``zeros_to_ncontig`` converts bit-exactly.
  w = (q - zp) * s with zp = 2 when no zeros are given (gemv/moe_gemv_int2_tab.py:66).
"""
from __future__ import annotations

import math
import os
import time

import torch

GROUP = 128

__all__ = [
    "pack_2bit_along_last", "pack_words_along_k", "to_word_ncontig", "unpack_words",
    "pack_zeros", "zeros_to_ncontig", "unpack_zeros_nc", "dequant", "gemv_tab", "gemv_byte_tab",
    "route_topk", "moe_layer", "moe_layer_routed_only", "moe_layer_by_expert", "int8_pack", "int8_unpack", "int8_gemv",
    "bf16_round", "max_rel_err", "norm_rel_err", "time_cpu_layer", "cpu_info", "routed_experts_from_arena",
    "moe_layer_from_arena",
]


# ----------------------------------------------------------------------------- packing / layout
def pack_2bit_along_last(q: torch.Tensor) -> torch.Tensor:
    """int [..., K] in 0..3 -> uint8 [..., K/4], value k at bits 2*(k%4) of byte k//4.

    The moe_wna16 byte layout (series-0002:1920-1925; unpack rule serving patch:297-385)."""
    q = q.to(torch.int32)
    b = q[..., 0::4] | (q[..., 1::4] << 2) | (q[..., 2::4] << 4) | (q[..., 3::4] << 6)
    return b.to(torch.uint8)


def pack_words_along_k(q: torch.Tensor) -> torch.Tensor:
    """int [..., K] in 0..3 -> int32 [..., K/16], value k at bits 2*(k%16) (series-0002:1928-1933)."""
    q = q.to(torch.int64) & 0x3
    shifts = (2 * torch.arange(16, dtype=torch.int64))
    w = (q.reshape(*q.shape[:-1], q.shape[-1] // 16, 16) << shifts).sum(-1)
    # sum of disjoint bit fields == OR; fold into the signed int32 range
    w = torch.where(w >= 2**31, w - 2**32, w)
    return w.to(torch.int32)


def to_word_ncontig(qweight_u8_nk: torch.Tensor) -> torch.Tensor:
    """Loader layout uint8 [E, N, K/4] -> int32 [E, K/16, N] (gemv/moe_gemv_int2_tab.py:100-109).

    Byte kb of row n becomes byte kb%4 of word kb//4 at column n (little endian), so value k ends at
    bits 2*(k%16) of word k//16. Pure re-arrangement of the same bytes."""
    E, N, KB = qweight_u8_nk.shape
    assert KB % 4 == 0, KB
    t = qweight_u8_nk.permute(0, 2, 1).reshape(E, KB // 4, 4, N).permute(0, 1, 3, 2)
    return t.contiguous().view(torch.int32).reshape(E, KB // 4, N)


def unpack_words(w32: torch.Tensor) -> torch.Tensor:
    """int32 [..., K/16, N] -> int32 codes [..., K, N] (gemv/test_gemv_tab.py:39-44)."""
    *lead, KW, N = w32.shape
    q = torch.empty(*lead, KW, 16, N, dtype=torch.int32)
    for j in range(16):
        q[..., j, :] = (w32 >> (2 * j)) & 0x3
    return q.reshape(*lead, KW * 16, N)


def pack_zeros(zp: torch.Tensor) -> torch.Tensor:
    """Per-group zero points int [E, N, K/g] in 0..3 -> uint8 [E, N/4, K/g], the loader form.

    Zero point of column n at bits 2*(n%4) of byte n//4 (series-0002:1946-1947)."""
    return pack_2bit_along_last(zp.transpose(1, 2)).transpose(1, 2).contiguous()


def zeros_to_ncontig(qzeros: torch.Tensor) -> torch.Tensor:
    """Loader form uint8 [E, N/4, K/g] -> GEMV form uint8 [E, K/g, N/4] (transpose, same bytes)."""
    return qzeros.transpose(1, 2).contiguous()


def unpack_zeros_nc(qz_nc: torch.Tensor) -> torch.Tensor:
    """uint8 [..., G, N/4] -> int32 [..., G, N]; column n at bits 2*(n%4) of byte n//4.

    Same bit rule as the tiled kernel's zero-point branch (serving patch:235-245)."""
    b = qz_nc.to(torch.int32)
    z = torch.stack([(b >> (2 * i)) & 0x3 for i in range(4)], dim=-1)
    return z.reshape(*qz_nc.shape[:-1], qz_nc.shape[-1] * 4)


def dequant(w32: torch.Tensor, scales: torch.Tensor, zeros_nc: torch.Tensor | None = None,
            group: int = GROUP) -> torch.Tensor:
    """Dequantize to fp32 [..., K, N]: (q - zp) * s, zp = 2 when ``zeros_nc`` is None.

    Symmetric form: gemv/test_gemv_tab.py:39-44 and series-0002:1976-1981; per-group zero point:
    series-0002:1936-1954 and the tiled kernel's dequant (serving patch:269-272)."""
    q = unpack_words(w32).float()
    s = scales.float().repeat_interleave(group, dim=-2)
    if zeros_nc is None:
        return (q - 2.0) * s
    z = unpack_zeros_nc(zeros_nc).float().repeat_interleave(group, dim=-2)
    return (q - z) * s


# ----------------------------------------------------------------------------- GEMV semantics
def gemv_tab(a: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, ids: torch.Tensor,
             topk_w: torch.Tensor | None, top_k: int, mul_routed_weight: bool,
             zeros_nc: torch.Tensor | None = None, slots: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 [R, N] result of ``moe_gemv_int2_tab`` (gemv/moe_gemv_int2_tab.py:23-69).

    Row r reads activation row r // top_k (:51) and expert e = ids[r] (:39); the routed weight
    multiplies the row when ``mul_routed_weight`` (:67-68). ``slots`` (int32 [E]) is the arena
    indirection of this build: codes/scales/zeros are then indexed by slot, and slot -1 gives a
    zero row (the reference has no mask; its tables always hold an address, gemv/expert_elastic.py)."""
    a = a.float()
    R = ids.numel()
    out = torch.zeros(R, codes.shape[-1], dtype=torch.float32)
    for r in range(R):
        e = int(ids[r])
        if slots is not None:
            e = int(slots[e])
            if e < 0:
                continue
        W = dequant(codes[e], scales[e], None if zeros_nc is None else zeros_nc[e])   # [K, N]
        v = a[r // top_k] @ W
        if mul_routed_weight:
            v = v * float(topk_w[r])
        out[r] = v
    return out


def gemv_byte_tab(x: torch.Tensor, qweight_nk4: torch.Tensor, scales_nk: torch.Tensor,
                  eids: torch.Tensor) -> torch.Tensor:
    """fp32 [T, N] result of the byte-layout GEMV ``gemv_int2`` (gemv/moe_gemv_int2.py:23-61).

    qweight uint8 [E, N, K/4] (value k at bits 2*(k%4) of byte k//4), scales f16 [E, N, K/128],
    symmetric zero point 2; x [K] shared or [T, K] per row (:64-71)."""
    T = eids.numel()
    out = torch.zeros(T, qweight_nk4.shape[1], dtype=torch.float32)
    for t in range(T):
        e = int(eids[t])
        b = qweight_nk4[e].to(torch.int32)                                  # [N, K/4]
        q = torch.stack([(b >> (2 * j)) & 3 for j in range(4)], dim=-1).reshape(b.shape[0], -1)
        W = (q.float() - 2.0) * scales_nk[e].float().repeat_interleave(GROUP, dim=1)    # [N, K]
        xv = x.float() if x.dim() == 1 else x[t].float()
        out[t] = W @ xv
    return out


# ----------------------------------------------------------------------------- routing
def route_topk(logits: torch.Tensor, k: int, renormalize: bool = True):
    """Softmax over fp32 logits, top-k, optional renormalisation -> (ids int32 [M,k], w fp32 [M,k]).

    The router the synthetic MoE test compares against (series-0002:1962-1965)
    ask for the renormalised form."""
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(p, k, dim=-1)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return ids.to(torch.int32), w.float()


# ----------------------------------------------------------------------------- full decode layer
def _silu(v: torch.Tensor) -> torch.Tensor:
    return v / (1.0 + torch.exp(-v))


def moe_layer(x: torch.Tensor, w13: torch.Tensor, s13: torch.Tensor, w2: torch.Tensor,
              s2: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor,
              z13: torch.Tensor | None = None, z2: torch.Tensor | None = None,
              routed_scaling_factor: float = 1.0, slots: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 [M, H]: sum_j w[m,j] * down_e(silu(gate_e(x_m)) * up_e(x_m)), e = topk_ids[m, j].

    The reference's fp32 layer reference (gemv/test_gemv_tab.py:73-76) generalised to M tokens and
    the composite ``_apply_gemv`` (patches/ncontig_gemv.py:218-238: gate_up GEMV, SiLU*mul with gate =
    rows [0, I) and up = rows [I, 2I), down GEMV times the routed weight, sum over top-k, times
    routed_scaling_factor). Expert tensors are indexed by ``slots[e]`` when given; slot -1 masks."""
    M, k = topk_ids.shape
    I = w13.shape[-1] // 2
    H = w2.shape[-1]
    y = torch.zeros(M, H, dtype=torch.float32)
    cache = {}
    for m in range(M):
        xm = x[m].float()
        for j in range(k):
            e = int(topk_ids[m, j])
            if slots is not None:
                e = int(slots[e])
                if e < 0:
                    continue
            if e not in cache:
                cache[e] = (dequant(w13[e], s13[e], None if z13 is None else z13[e]),
                            dequant(w2[e], s2[e], None if z2 is None else z2[e]))
            W13, W2 = cache[e]
            gu = xm @ W13                                  # [2I]
            h = _silu(gu[:I]) * gu[I:]
            y[m] += float(topk_w[m, j]) * (h @ W2)
    return y * float(routed_scaling_factor)


def moe_layer_routed_only(x, experts_cpu: dict, topk_ids, topk_w, routed_scaling_factor=1.0):
    """Same math as :func:`moe_layer`, but the expert tensors are a dict e -> (w13, s13, z13, w2,
    s2, z2) holding only the routed experts (what a timed CPU baseline copies off the device).
    Experts absent from the dict count as masked (slot -1)."""
    M, k = topk_ids.shape
    y = None
    for m in range(M):
        xm = x[m].float()
        for j in range(k):
            e = int(topk_ids[m, j])
            if e not in experts_cpu:
                continue
            w13, s13, z13, w2, s2, z2 = experts_cpu[e]
            W13 = dequant(w13, s13, z13)
            W2 = dequant(w2, s2, z2)
            I = W13.shape[-1] // 2
            gu = xm @ W13
            h = _silu(gu[:I]) * gu[I:]
            d = float(topk_w[m, j]) * (h @ W2)
            if y is None:
                y = torch.zeros(M, d.shape[-1], dtype=torch.float32)
            y[m] += d
    return None if y is None else y * float(routed_scaling_factor)   # None: no routed expert is present


def routed_experts_from_arena(arena, ids) -> dict:
    """Copy the routed experts of an arena-like object (attributes slots, codes13, scales13, zeros13,
    codes2, scales2, zeros2; device tensors) to the host, keyed by expert id; slot -1 is skipped."""
    slots = arena.slots.cpu()
    experts = {}
    for e in sorted(set(ids.cpu().reshape(-1).tolist())):
        sl = int(slots[e])
        if sl < 0:
            continue
        pick = lambda t: None if t is None else t[sl].cpu()
        experts[e] = (pick(arena.codes13), pick(arena.scales13), pick(arena.zeros13),
                      pick(arena.codes2), pick(arena.scales2), pick(arena.zeros2))
    return experts


def moe_layer_by_expert(arena, x, topk_ids, topk_w, routed_scaling_factor: float = 1.0) -> torch.Tensor:
    """fp32 [M, H]: the math of :func:`moe_layer_routed_only` (the reference's fp32 layer,
    gemv/test_gemv_tab.py:73-76, with the composite of patches/ncontig_gemv.py:218-238) in expert order:
    each distinct routed, resident expert is copied off the device and dequantised once and applied to
    every token routed to it, so whole batches of tokens at full size can be checked. Per token the top-k
    contributions are added in routing order, as in the token-order loop."""
    M = x.shape[0]
    ids = topk_ids.cpu().reshape(M, -1)
    w = topk_w.cpu().reshape(M, -1)
    k = ids.shape[1]
    slots = arena.slots.cpu()
    xs = x.cpu().float()
    H = xs.shape[1]
    contrib = torch.zeros(M, k, H, dtype=torch.float32)
    for e in sorted(set(ids.reshape(-1).tolist())):
        sl = int(slots[e]) if 0 <= e < slots.numel() else -1
        if sl < 0 or sl >= arena.codes13.shape[0]:
            continue
        pick = lambda t: None if t is None else t[sl].cpu()
        W13 = dequant(pick(arena.codes13), pick(arena.scales13), pick(arena.zeros13))
        W2 = dequant(pick(arena.codes2), pick(arena.scales2), pick(arena.zeros2))
        I = W13.shape[-1] // 2
        where = (ids == e).nonzero().tolist()
        toks = sorted({m for m, _ in where})
        gu = xs[toks] @ W13                                  # [t, 2I]
        h = _silu(gu[:, :I]) * gu[:, I:]
        yd = h @ W2                                          # [t, H]
        row = {m: i for i, m in enumerate(toks)}
        for m, j in where:
            contrib[m, j] = float(w[m, j]) * yd[row[m]]
    y = torch.zeros(M, H, dtype=torch.float32)
    for j in range(k):
        y += contrib[:, j]
    return y * float(routed_scaling_factor)


def moe_layer_from_arena(arena, x, topk_ids, topk_w, routed_scaling_factor: float = 1.0) -> torch.Tensor:
    """fp32 oracle of the decode layer for an arena-like object (see routed_experts_from_arena)."""
    experts = routed_experts_from_arena(arena, topk_ids)
    ids = topk_ids.cpu().reshape(x.shape[0], -1)
    w = topk_w.cpu().reshape(x.shape[0], -1)
    y = moe_layer_routed_only(x.cpu(), experts, ids, w, routed_scaling_factor)
    return torch.zeros(x.shape, dtype=torch.float32) if y is None else y


# ----------------------------------------------------------------------------- INT8 dense GEMV
def int8_pack(q_u8_kn: torch.Tensor) -> torch.Tensor:
    """uint8-valued int [K, N] (0..255) -> int32 [K/4, N], byte i of word kb = value 4*kb + i.

    The auto_gptq INT8 packing of scripts/requant_int8.py:32-50 (4 values per int32 along K,
    little-endian, shift 8*(k%4))."""
    K, N = q_u8_kn.shape
    q = q_u8_kn.to(torch.int64) & 0xFF
    w = q[0::4] | (q[1::4] << 8) | (q[2::4] << 16) | (q[3::4] << 24)
    w = torch.where(w >= 2**31, w - 2**32, w)
    return w.to(torch.int32).contiguous()


def int8_unpack(qw: torch.Tensor) -> torch.Tensor:
    """int32 [K/4, N] -> int32 [K, N] in 0..255 (scripts/requant_int8.py:53-58)."""
    KW, N = qw.shape
    q = torch.empty(KW, 4, N, dtype=torch.int32)
    for i in range(4):
        q[:, i, :] = (qw >> (8 * i)) & 0xFF
    return q.reshape(KW * 4, N)


def int8_gemv(x: torch.Tensor, qw: torch.Tensor, scales: torch.Tensor, zero: int = 128) -> torch.Tensor:
    """fp32 [M, N] = x @ ((q - zero) * s) with q from ``int8_unpack``; ``scales`` f16 [K/g, N]
    (g = K / scales.shape[0]; one row = per-output-channel). Dequant rule of
    scripts/requant_int8.py:53-63 (zero 128 symmetric, stored as 127 + 1)."""
    q = int8_unpack(qw).float()
    K = q.shape[0]
    g = K // scales.shape[0]
    W = (q - float(zero)) * scales.float().repeat_interleave(g, dim=0)
    xx = x.float() if x.dim() == 2 else x.float()[None]
    return xx @ W


# ----------------------------------------------------------------------------- comparison helpers
def bf16_round(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


def max_rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max |got - ref| / max |ref| (the max-relative-error bar used by the tests)."""
    got, ref = got.float(), ref.float()
    den = ref.abs().max().item()
    return (got - ref).abs().max().item() / (den if den > 0 else 1.0)


def norm_rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """||got - ref|| / ||ref|| (the reference tests' measure, gemv/test_gemv_tab.py:80)."""
    got, ref = got.float(), ref.float()
    den = ref.norm().item()
    return (got - ref).norm().item() / (den if den > 0 else 1.0)


# ----------------------------------------------------------------------------- CPU timing
def cpu_info() -> dict:
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(), "cpu_model": model}


def time_cpu_layer(x, experts_cpu, topk_ids, topk_w, budget_s: float = 10.0, min_iters: int = 1):
    """Time :func:`moe_layer_routed_only` (the reference formulation: dequantize the routed experts
    in fp32, then the matmuls) with all host threads; returns (seconds per layer, iterations)."""
    torch.set_num_threads(os.cpu_count() or 1)
    moe_layer_routed_only(x, experts_cpu, topk_ids, topk_w)          # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        moe_layer_routed_only(x, experts_cpu, topk_ids, topk_w)
        n += 1
        el = time.perf_counter() - t0
        if n >= min_iters and el >= budget_s:
            break
        if n >= min_iters and el / n * (n + 1) > budget_s * 1.5:
            break
    return el / n, n
