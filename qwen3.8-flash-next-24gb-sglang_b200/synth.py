"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configurations.

No checkpoint or dataset is involved: codes are uniform 2-bit values (random 32-bit words hold 16
independent uniform codes), scales are |N(0,1)| * 0.02 in f16, per-group zero points are uniform
in {0..3}, activations bf16 ~ N(0,1), router logits fp32 ~ N(0,1) (softmax -> top-k ->
renormalise). Config 2's residency follows a Zipf(s) expert popularity; config 3 uses uniform
random logits.
"""
from __future__ import annotations

import math

import torch

from .moe_layer import ExpertArena

__all__ = ["gen", "random_words", "make_arena", "make_activation", "route_softmax", "route_zipf",
           "zipf_popularity", "resident_slots", "make_int8_dense", "ROUTED_SCALING"]

ROUTED_SCALING = 1.0


def gen(seed: int, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def random_words(shape, g: torch.Generator, device="cpu") -> torch.Tensor:
    """int32 words with uniform random bits = 16 independent uniform 2-bit codes each."""
    return torch.randint(-(2 ** 31), 2 ** 31, tuple(shape), dtype=torch.int32, generator=g, device=device)


def _scales(shape, g, device, dtype):
    return (torch.randn(tuple(shape), generator=g, device=device).abs() * 0.02).to(dtype)


def make_arena(S: int, H: int, I: int, *, seed: int = 0, zeros: bool = True, scale_dtype=torch.float16,
               device="cuda", gen_device=None, slots: torch.Tensor | None = None) -> ExpertArena:
    """S experts of one layer: gate_up [2I, H] and down [H, I] in the word layout, on ``device``.
    ``gen_device`` chooses where the random numbers are drawn (CPU for bit-reproducible test data)."""
    gd = device if gen_device is None else gen_device
    g = gen(seed, gd)
    c13 = random_words((S, H // 16, 2 * I), g, gd)
    s13 = _scales((S, H // 128, 2 * I), g, gd, scale_dtype)
    c2 = random_words((S, I // 16, H), g, gd)
    s2 = _scales((S, I // 128, H), g, gd, scale_dtype)
    z13 = z2 = None
    if zeros:
        z13 = torch.randint(0, 256, (S, H // 128, (2 * I) // 4), dtype=torch.uint8, generator=g, device=gd)
        z2 = torch.randint(0, 256, (S, I // 128, H // 4), dtype=torch.uint8, generator=g, device=gd)
    mv = lambda t: None if t is None else t.to(device).contiguous()
    return ExpertArena(mv(c13), mv(s13), mv(c2), mv(s2), mv(z13), mv(z2),
                       None if slots is None else slots.to(device=device, dtype=torch.int32))


def make_activation(M: int, H: int, *, seed: int = 0, device="cuda", gen_device=None) -> torch.Tensor:
    gd = device if gen_device is None else gen_device
    return torch.randn((M, H), generator=gen(seed + 7, gd), device=gd).to(torch.bfloat16).to(device)


def route_softmax(M: int, E: int, top_k: int, *, seed: int = 0, device="cuda", gen_device=None,
                  uniform_logits: bool = False, renormalize: bool = True):
    """Router: fp32 logits ~ N(0,1) (or U(0,1)), softmax, top-k, renormalise -> (ids int32, w fp32)."""
    gd = device if gen_device is None else gen_device
    g = gen(seed + 11, gd)
    logits = (torch.rand((M, E), generator=g, device=gd) if uniform_logits
              else torch.randn((M, E), generator=g, device=gd))
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(p, top_k, dim=-1)
    if renormalize:
        w = w / w.sum(-1, keepdim=True)
    return ids.to(torch.int32).to(device), w.float().to(device)


def zipf_popularity(E: int, s: float = 1.1, *, seed: int = 0) -> torch.Tensor:
    """fp32 [E] popularity: rank r (1-based) has weight r^-s; ranks assigned by a seeded permutation."""
    g = gen(seed + 13)
    perm = torch.randperm(E, generator=g)
    w = torch.arange(1, E + 1, dtype=torch.float64).pow(-s)
    p = torch.empty(E, dtype=torch.float64)
    p[perm] = w
    return (p / p.sum()).float()


def route_zipf(M: int, E: int, top_k: int, pop: torch.Tensor, *, seed: int = 0, device="cuda"):
    """top-k experts per token sampled without replacement from ``pop`` (Gumbel top-k); weights are a
    softmax of N(0,1) logits over the chosen experts."""
    g = gen(seed + 17)
    gumbel = -torch.log(-torch.log(torch.rand((M, E), generator=g).clamp_min(1e-12)))
    ids = torch.topk(torch.log(pop.double())[None, :] + gumbel.double(), top_k, dim=-1).indices
    w = torch.softmax(torch.randn((M, top_k), generator=g), dim=-1)
    return ids.to(torch.int32).to(device), w.float().to(device)


def resident_slots(pop: torch.Tensor, S: int, *, seed: int = 0) -> torch.Tensor:
    """int32 [E] slot table: the S most popular experts (the hottest-S rule of patches/placement.py:114-116)
    get arena rows in a seeded random permutation; the rest get -1."""
    E = pop.numel()
    hot = torch.argsort(pop, descending=True)[:S]
    perm = torch.randperm(S, generator=gen(seed + 19))
    slots = torch.full((E,), -1, dtype=torch.int32)
    slots[hot] = perm.to(torch.int32)
    return slots


def make_int8_dense(K: int, N: int, *, seed: int = 0, device="cuda", gen_device=None):
    """INT8 dense projection [K -> N]: weights uniform in [-127, 127] stored as uint8 q = w + 128 packed
    4 per int32 along K ([K/4, N]), per-output-channel f16 scale |N(0,1)| * 0.005 (scales [1, N])."""
    gd = device if gen_device is None else gen_device
    g = gen(seed + 23, gd)
    wq = torch.randint(-127, 128, (K, N), dtype=torch.int32, generator=g, device=gd) + 128
    packed = (wq[0::4] | (wq[1::4] << 8) | (wq[2::4] << 16) | (wq[3::4] << 24))
    packed = packed.to(torch.int64)
    packed = torch.where(packed >= 2 ** 31, packed - 2 ** 32, packed).to(torch.int32)
    scales = (torch.randn((1, N), generator=g, device=gd).abs() * 0.005).to(torch.float16)
    return packed.to(device).contiguous(), scales.to(device).contiguous()
