"""GPU parity of the batched decode layer -- M >= 16 tokens: the routed rows grouped by expert, every resident
expert streamed once for all of its rows, the products on the tensor cores -- against the fp32 CPU oracle with
every token checked, and against the per-token layer (the int64-table entry point, which always takes it) on
the same inputs. Bar: max relative error <= 1e-2 on bf16 outputs, as for the per-token layer."""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def per_token(pkg, arena, x, ids, w, rsf):
    """The same layer through the table form (per-token fused path, any M)."""
    wt13, st13, sw13, ss13 = pkg.make_tables(arena.codes13, arena.scales13)
    wt2, st2, sw2, ss2 = pkg.make_tables(arena.codes2, arena.scales2)
    zt = (pkg.make_zero_table(arena.zeros13)[0], pkg.make_zero_table(arena.zeros2)[0]) if arena.zeros13 is not None \
        else None
    # the tables index experts directly: route through the slot table first (masked experts -> weight 0)
    sl = arena.slots[ids.long()]
    ids_s = sl.clamp_min(0).to(torch.int32)
    w_s = torch.where(sl >= 0, w, torch.zeros_like(w))
    H, I = arena.H, arena.I
    tabs = ((wt13, st13, sw13, ss13), (wt2, st2, sw2, ss2), 2 * I, H, H, I, arena.scale_bf16)
    return pkg.apply_gemv(x, ids_s, w_s, tabs, rsf, zero_tabs=zt)


@pytest.mark.parametrize("M,E,H,I,k,zeros,sdt,rsf", [
    (16, 8, 256, 256, 4, True, torch.float16, 1.0),
    (40, 16, 512, 384, 8, False, torch.bfloat16, 2.5),
    (150, 32, 1024, 512, 8, True, torch.bfloat16, 1.0),    # three launches of up to 64 tokens
])
def test_batched_layer_vs_oracle_and_per_token(pkg, dev, M, E, H, I, k, zeros, sdt, rsf):
    arena = pkg.synth.make_arena(E, H, I, seed=M, zeros=zeros, scale_dtype=sdt, device=dev, gen_device="cpu")
    x = pkg.synth.make_activation(M, H, seed=M, device=dev, gen_device="cpu")
    ids, w = pkg.synth.route_softmax(M, E, k, seed=M, device=dev, gen_device="cpu")
    y = pkg.moe_decode_layer(x, ids, w, arena, routed_scaling_factor=rsf, batched=True)
    torch.cuda.synchronize()
    ref = O.moe_layer_from_arena(arena, x, ids, w, rsf)
    err = O.max_rel_err(y.float().cpu(), ref)
    assert err < TOL, err
    y_pt = per_token(pkg, arena, x, ids, w, rsf)
    err_pt = O.max_rel_err(y.float().cpu(), y_pt.float().cpu())
    assert err_pt < TOL, err_pt
    # deterministic: a second call gives the same bits
    assert torch.equal(pkg.moe_decode_layer(x, ids, w, arena, routed_scaling_factor=rsf, batched=True), y)


def test_batched_layer_skewed_and_masked(pkg, dev):
    """One expert takes every token (48 rows: three groups of 16), two experts are not resident (slot -1), and
    the arena order differs from the expert order."""
    M, E, H, I, k = 48, 8, 256, 256, 2
    slots = torch.tensor([3, 0, 5, 1, 2, -1, -1, 4], dtype=torch.int32)
    arena = pkg.synth.make_arena(6, H, I, seed=11, zeros=True, device=dev, gen_device="cpu", slots=slots)
    x = pkg.synth.make_activation(M, H, seed=11, device=dev, gen_device="cpu")
    m = torch.arange(M)
    ids = torch.stack([torch.zeros(M, dtype=torch.long), 1 + m % 7], 1).to(torch.int32).to(dev)
    w = torch.rand((M, k), generator=torch.Generator().manual_seed(11)).add_(0.1).to(dev)
    y = pkg.moe_decode_layer(x, ids, w, arena, batched=True)
    torch.cuda.synchronize()
    ref = O.moe_layer_from_arena(arena, x, ids, w, 1.0)
    err = O.max_rel_err(y.float().cpu(), ref)
    assert err < TOL, err
    # masking == zero routing weight, through the same batched path
    hit = arena.slots[ids.long()] >= 0
    y0 = pkg.moe_decode_layer(x, ids, torch.where(hit, w, torch.zeros_like(w)), arena, batched=True)
    assert torch.equal(y0, y)


def test_batched_and_per_token_calls_share_the_workspace(pkg, dev):
    """The batched path never writes the per-token path's persistent workspace words (grid-barrier counters,
    epoch-tagged hand-off words): per-token and batched calls alternating on the one shared workspace all stay
    correct."""
    E, H, I, k = 16, 512, 256, 4
    arena = pkg.synth.make_arena(E, H, I, seed=21, zeros=True, device=dev, gen_device="cpu")
    for j, M in enumerate((1, 16, 2, 40, 1, 16, 1)):
        x = pkg.synth.make_activation(M, H, seed=21 + j, device=dev, gen_device="cpu")
        ids, w = pkg.synth.route_softmax(M, E, k, seed=21 + j, device=dev, gen_device="cpu")
        y = pkg.moe_decode_layer(x, ids, w, arena, batched=M >= 16)
        torch.cuda.synchronize()
        err = O.max_rel_err(y.float().cpu(), O.moe_layer_from_arena(arena, x, ids, w, 1.0))
        assert err < TOL, (j, M, err)
