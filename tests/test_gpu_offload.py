"""The caller's side of the path on a GPU: the load-time relayout of device and host (pinned or pageable)
tensors, MoeWNA16Method's dispatch (the M <= 16 GEMV branch and the tiled branch), and experts that live in
pinned host memory read through the int64 address tables (the reference's offloaded layers,
gemv/moe_gemv_int2_tab.py:12-14, test_gemv_tab.py:78-92). Bars as elsewhere: relayout bit-exact, bf16
outputs within max relative error 1e-2 of the fp32 oracle."""
from types import SimpleNamespace

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def test_relayout_of_host_tensors(pkg, dev):
    """to_word_ncontig of a pinned tensor returns a pinned tensor, of a pageable one a pinned tensor too,
    both bit-identical to the oracle's relayout (the CUDA kernel reads and writes host memory)."""
    g = torch.Generator().manual_seed(41)
    src = torch.randint(0, 256, (3, 96, 64), dtype=torch.uint8, generator=g)
    ref = O.to_word_ncontig(src)
    for t in (src.pin_memory(), src.clone()):
        out = pkg.to_word_ncontig(t)
        assert not out.is_cuda and out.is_pinned()
        assert torch.equal(out, ref)
    assert torch.equal(pkg.to_word_ncontig(src.to(dev)).cpu(), ref)


def _loader_layer(E, H, I, seed, device, zeros=True, sdt=torch.bfloat16, pin=False):
    """A layer as the checkpoint loader leaves it: codes uint8 [E, N, K/4], scales [E, N, K/128], zero points
    uint8 [E, N/4, K/128] (series-0002:1920-1954)."""
    g = torch.Generator().manual_seed(seed)
    mk = lambda *sh: torch.randint(0, 256, sh, dtype=torch.uint8, generator=g)
    sc = lambda *sh: (torch.randn(*sh, generator=g).abs() * 0.02).to(sdt)
    t = dict(w13_qweight=mk(E, 2 * I, H // 4), w2_qweight=mk(E, H, I // 4),
             w13_scales=sc(E, 2 * I, H // 128), w2_scales=sc(E, H, I // 128))
    if zeros:
        t.update(w13_qzeros=mk(E, 2 * I // 4, H // 128), w2_qzeros=mk(E, H // 4, I // 128))
    put = (lambda x: x.pin_memory()) if pin else (lambda x: x.to(device))
    return SimpleNamespace(**{k: put(v) for k, v in t.items()})


def _oracle(layer, x, ids, w, rsf):
    arena = SimpleNamespace(codes13=layer.w13_qweight, scales13=layer.w13_scales, codes2=layer.w2_qweight,
                            scales2=layer.w2_scales, zeros13=getattr(layer, "w13_qzeros", None),
                            zeros2=getattr(layer, "w2_qzeros", None),
                            slots=torch.arange(layer.w13_qweight.shape[0], dtype=torch.int32))
    return O.moe_layer_by_expert(arena, x, ids, w, rsf)


@pytest.mark.parametrize("M", [1, 16, 20, 64])
def test_method_dispatch_on_device(pkg, dev, M):
    """process_weights_after_loading then apply: at most 16 tokens through the GEMV composite, more through
    the tiled branch; every token against the oracle."""
    E, H, I, k = 16, 1024, 512, 4
    layer = _loader_layer(E, H, I, seed=M, device=dev)
    meth = pkg.MoeWNA16Method(routed_scaling_factor=1.5)
    meth.process_weights_after_loading(layer)
    assert layer._b_n_contig and layer.w13_qweight.shape == (E, H // 16, 2 * I)
    assert layer.w13_scales.shape == (E, H // 128, 2 * I) and layer.w13_qzeros.shape == (E, H // 128, 2 * I // 4)
    x = pkg.synth.make_activation(M, H, seed=M, device=dev, gen_device="cpu")
    ids, w = pkg.synth.route_softmax(M, E, k, seed=M, device=dev, gen_device="cpu")
    y = meth.apply(layer, x, ids, w)
    torch.cuda.synchronize()
    assert (layer._gemv_tabs is not None) == (M <= 16)
    ref = _oracle(layer, x, ids, w, 1.5)
    assert O.max_rel_err(y.float().cpu(), ref) < TOL


def test_offloaded_layer_reads_pinned_host_experts(pkg, dev):
    """A layer whose experts stay in pinned host memory (the reference's offloaded layers): the relayout keeps
    them pinned, the table entries hold host addresses, and the GEMV branch reads the experts over the bus."""
    E, H, I, k, M = 8, 1024, 512, 4, 2
    layer = _loader_layer(E, H, I, seed=3, device=dev, pin=True)
    meth = pkg.MoeWNA16Method()
    meth.process_weights_after_loading(layer)
    for n in ("w13_qweight", "w2_qweight", "w13_scales", "w2_scales", "w13_qzeros", "w2_qzeros"):
        t = getattr(layer, n)
        assert not t.is_cuda and t.is_pinned(), n
    x = pkg.synth.make_activation(M, H, seed=3, device=dev, gen_device="cpu")
    ids, w = pkg.synth.route_softmax(M, E, k, seed=3, device=dev, gen_device="cpu")
    y = meth.apply(layer, x, ids, w)
    torch.cuda.synchronize()
    assert int(layer._gemv_tabs[0][0][0]) == layer.w13_qweight.data_ptr()      # a host address in the table
    assert O.max_rel_err(y.float().cpu(), _oracle(layer, x, ids, w, 1.0)) < TOL


def test_mixed_device_and_host_table_entries(pkg, dev):
    """moe_gemv_int2_tab and the fused layer through tables whose entries point some experts at device
    memory and the others at pinned host memory (the elastic placement's table, gemv/expert_elastic.py:157):
    results equal the all-device tables bit for bit."""
    E, H, I, k, M = 8, 1024, 512, 4, 2
    arena = pkg.synth.make_arena(E, H, I, seed=5, zeros=True, device=dev, gen_device="cpu")
    host = {n: getattr(arena, n).cpu().pin_memory() for n in ("codes13", "scales13", "zeros13", "codes2",
                                                             "scales2", "zeros2")}
    on_host = torch.tensor([e % 2 == 1 for e in range(E)])

    def tab(name):
        d, h = getattr(arena, name), host[name]
        rb = d[0].numel() * d.element_size()
        addr = [(h.data_ptr() if on_host[e] else d.data_ptr()) + e * rb for e in range(E)]
        return torch.tensor(addr, dtype=torch.int64, device=dev)

    x = pkg.synth.make_activation(M, H, seed=5, device=dev, gen_device="cpu")
    ids, w = pkg.synth.route_softmax(M, E, k, seed=5, device=dev, gen_device="cpu")
    wt, st, sw, ss = pkg.make_tables(arena.codes13, arena.scales13)
    zt, zg = pkg.make_zero_table(arena.zeros13)
    ref = pkg.moe_gemv_int2_tab(x, wt, st, ids.reshape(-1), w.reshape(-1), 2 * I, H, sw, ss, k, False,
                                scale_bf16=False, ztab=zt, stride_zg=zg)
    got = pkg.moe_gemv_int2_tab(x, tab("codes13"), tab("scales13"), ids.reshape(-1), w.reshape(-1), 2 * I, H, sw,
                                ss, k, False, scale_bf16=False, ztab=tab("zeros13"), stride_zg=zg)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    tabs_dev = (pkg.make_tables(arena.codes13, arena.scales13), pkg.make_tables(arena.codes2, arena.scales2),
                2 * I, H, H, I, False)
    zdev = (pkg.make_zero_table(arena.zeros13)[0], pkg.make_zero_table(arena.zeros2)[0])
    tabs_mix = ((tab("codes13"), tab("scales13"), sw, ss), (tab("codes2"), tab("scales2"), H, H), 2 * I, H, H, I,
                False)
    y_dev = pkg.apply_gemv(x, ids, w, tabs_dev, None, zero_tabs=zdev)
    y_mix = pkg.apply_gemv(x, ids, w, tabs_mix, None, zero_tabs=(tab("zeros13"), tab("zeros2")))
    torch.cuda.synchronize()
    assert torch.equal(y_mix, y_dev)
    assert O.max_rel_err(y_mix.float().cpu(), O.moe_layer_from_arena(arena, x, ids, w)) < TOL
