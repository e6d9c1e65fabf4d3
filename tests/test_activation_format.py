"""Error envelope of the kernels' activation format (the W2 layer and the INT8 projection), on the CPU (no kernel
runs here).

The kernels hold x in 16-bit block fixed point: per 128-value group, x16 = round(x / 2^e) clamped to +-32767,
with e the frexp exponent of the group's max |x| minus 15 (the activation tables of csrc/w2a16_common.cuh).
h = silu(gate) * up is held the same way per 32-value block (htab_block in csrc/w2a16_layer.cu). Codes times
fixed-point values are summed exactly in int32 per quantisation group, and the zero point and the group's scale
are folded in exactly. So, apart from fp32 accumulation across groups and the bf16 output, the format is the
kernels' only approximation. The layer evaluated in fp64 with x and h replaced by their fixed-point values is a
model of the kernels' arithmetic.

The GPU parity tests compare the kernels themselves with the oracle on N(0,1) activations. This test bounds the
format's own share of the error at config 1's full size (H=4096, I=1536, top-8 of 16 experts, per-group zero
points). It also covers activations with outlier channels, which the synthetic inputs lack. The bar is the tests'
1e-2; the format alone stays two orders of magnitude below it, so the bf16 rounding of the output dominates.
"""
import pytest
import torch
import torch.nn.functional as F

import oracle as O

TOL = 1e-2
FORMAT_TOL = 1e-3          # the format's own share (measured at most 1.6e-4 over the cases below)
BATCHED_FORMAT_TOL = 5e-3  # the batched path's (measured 1.7e-3, nearly all from h rounded to bf16)


def fixed_point(v: torch.Tensor, block: int, frac: int = 15) -> torch.Tensor:
    """The values the format represents v by (fp64): one exponent per `block` values, round half to even.
    frac 15: the per-token kernels (|x16| <= 32767); 14: the batched path (|x16| <= 2^14, split into bytes)."""
    b = v.reshape(-1, block).double()
    mx = b.abs().amax(dim=1, keepdim=True)
    _, ex = torch.frexp(mx)                                    # mx = f * 2^ex, f in [0.5, 1)
    e = torch.where(mx > 0, ex, torch.zeros_like(ex)) - frac
    step = torch.pow(2.0, e.double())
    return (torch.clamp(torch.round(b / step), -32767, 32767) * step).reshape(v.shape)


def _experts(pkg, E, H, I, seed):
    sy = pkg.synth
    g = sy.gen(seed)
    c13 = sy.random_words((E, H // 16, 2 * I), g)
    s13 = (torch.randn((E, H // 128, 2 * I), generator=g).abs() * 0.02).half()
    c2 = sy.random_words((E, I // 16, H), g)
    s2 = (torch.randn((E, I // 128, H), generator=g).abs() * 0.02).half()
    z13 = torch.randint(0, 256, (E, H // 128, (2 * I) // 4), dtype=torch.uint8, generator=g)
    z2 = torch.randint(0, 256, (E, I // 128, H // 4), dtype=torch.uint8, generator=g)
    return c13, s13, z13, c2, s2, z2


def _oracle_and_model(experts, x, ids, w, batched=False):
    """(fp32 oracle layer, fp64 layer with x and h in the kernels' format) for one token. batched: the batched
    path's format (xtab_kernel in csrc/w2a16_grouped.cu): 15-bit values, and h rounded to bf16 by the gate_up
    epilogue, then converted per 128-value group like x."""
    c13, s13, z13, c2, s2, z2 = experts
    I = s13.shape[-1] // 2
    xf = x.float()
    xq = fixed_point(xf, 128, 14 if batched else 15)
    ref = torch.zeros(c2.shape[-1], dtype=torch.float64)
    mod = torch.zeros_like(ref)
    for e, we in zip(ids.tolist(), w.tolist()):
        W13 = O.dequant(c13[e], s13[e], z13[e])
        W2 = O.dequant(c2[e], s2[e], z2[e])
        gu = xf @ W13
        ref += we * (F.silu(gu[:I]) * gu[I:] @ W2).double()
        gq = xq @ W13.double()
        hq = (F.silu(gq[:I]) * gq[I:]).float()                # the kernels form h in fp32
        if batched:
            mod += we * (fixed_point(hq.to(torch.bfloat16).float(), 128, 14) @ W2.double())
        else:
            mod += we * (fixed_point(hq, 32) @ W2.double())
    return ref.float(), mod


def test_fixed_point_is_exact_near_the_group_maximum():
    """Every bf16 value at least 2^-8 of its group's power-of-two bound is represented exactly."""
    g = torch.Generator().manual_seed(1)
    v = (torch.randn(64, 128, generator=g) * torch.pow(2.0, torch.randint(-20, 20, (64, 1), generator=g).float()))
    v = v.to(torch.bfloat16).float()
    fp = fixed_point(v, 128).float()
    _, ex = torch.frexp(v.abs().amax(dim=1, keepdim=True))
    near = v.abs() >= torch.pow(2.0, (ex - 8).float())
    assert near.any() and torch.equal(fp[near], v[near])
    # and no value moves by more than half a step of its group
    assert ((fp - v).abs() <= torch.pow(2.0, (ex - 16).float())).all()


@pytest.mark.parametrize("case", ["normal", "x100_16ch", "x1000_16ch", "x1000_1ch", "x1000_per_group"])
def test_activation_format_error_at_config1(pkg, case):
    E, H, I, k = 16, 4096, 1536, 8
    experts = _experts(pkg, E, H, I, seed=0)
    ids, w = pkg.synth.route_softmax(1, E, k, seed=0, device="cpu")
    x = pkg.synth.make_activation(1, H, seed=0, device="cpu").float()[0]
    if case == "x100_16ch" or case == "x1000_16ch":
        ch = torch.randperm(H, generator=torch.Generator().manual_seed(3))[:16]
        x[ch] *= 100.0 if case == "x100_16ch" else 1000.0
    elif case == "x1000_1ch":
        x[7] *= 1000.0
    elif case == "x1000_per_group":
        x[5::128] *= 1000.0                                    # every group's exponent set by an outlier
    x = x.to(torch.bfloat16)
    ref, mod = _oracle_and_model(experts, x, ids[0], w[0])
    assert O.max_rel_err(mod.float(), ref) < FORMAT_TOL
    assert O.max_rel_err(mod.float().to(torch.bfloat16), ref) < TOL


@pytest.mark.parametrize("case", ["normal", "x1000_per_group"])
def test_int8_activation_format_error(pkg, case):
    """The INT8 dense kernels convert x the same way (per 128-value group); the projection 4096 -> 4096 with x in
    that format stays within the same envelope of the fp32 oracle."""
    K = N = 4096
    qw, sc = pkg.synth.make_int8_dense(K, N, seed=0, device="cpu")
    x = pkg.synth.make_activation(1, K, seed=1, device="cpu").float()
    if case == "x1000_per_group":
        x[:, 9::128] *= 1000.0
    x = x.to(torch.bfloat16)
    ref = O.int8_gemv(x, qw, sc)
    W = (O.int8_unpack(qw).double() - 128.0) * sc.double()
    mod = fixed_point(x.float(), 128) @ W
    assert O.max_rel_err(mod.float(), ref) < FORMAT_TOL
    assert O.max_rel_err(mod.float().to(torch.bfloat16), ref) < TOL


@pytest.mark.parametrize("case", ["normal", "x1000_per_group"])
def test_batched_activation_format_error_at_config1(pkg, case):
    """The batched path's format (x and bf16 h, 15-bit per 128-value group) at config 1's size."""
    E, H, I, k = 16, 4096, 1536, 8
    experts = _experts(pkg, E, H, I, seed=0)
    ids, w = pkg.synth.route_softmax(1, E, k, seed=0, device="cpu")
    x = pkg.synth.make_activation(1, H, seed=0, device="cpu").float()[0]
    if case == "x1000_per_group":
        x[5::128] *= 1000.0
    x = x.to(torch.bfloat16)
    ref, mod = _oracle_and_model(experts, x, ids[0], w[0], batched=True)
    assert O.max_rel_err(mod.float(), ref) < BATCHED_FORMAT_TOL
    assert O.max_rel_err(mod.float().to(torch.bfloat16), ref) < TOL
