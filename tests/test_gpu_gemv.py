"""GPU parity of the single GEMV entry points (moe_gemv_int2_tab / slots / relayout / gather)
against the CPU oracle and the reference's golden vectors. Bar: bf16 outputs within max relative
error 1e-2 of the fp32 oracle (the reference's own GEMV bar, series-0002:2231-2232); integer work
(relayout, gather, slot routing) bit-exact."""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _cuda(*ts, dev):
    return [None if t is None else t.to(dev) for t in ts]


def test_gemv_tab_matches_golden_reference_outputs(pkg, golden, dev):
    for s in ("f16", "bf16"):
        g = lambda k: golden[f"tab_{s}_{k}"]
        w13, s13, w2, s2 = _cuda(g("w13"), g("s13"), g("w2"), g("s2"), dev=dev)
        wt13, st13, sw13, ss13 = pkg.make_tables(w13, s13)
        wt2, st2, sw2, ss2 = pkg.make_tables(w2, s2)
        ids, rw = g("ids").to(dev), g("rw").to(dev)
        sbf = s == "bf16"
        o13 = pkg.moe_gemv_int2_tab(g("x13").to(dev), wt13, st13, ids, rw, 200, 256, sw13, ss13, top_k=3,
                                    mul_routed_weight=False, scale_bf16=sbf)
        o2 = pkg.moe_gemv_int2_tab(g("x2").to(dev), wt2, st2, ids, rw, 256, 128, sw2, ss2, top_k=1,
                                   mul_routed_weight=True, scale_bf16=sbf)
        torch.cuda.synchronize()
        assert o13.shape == (3, 200) and o13.dtype == torch.bfloat16 and o2.shape == (3, 256)
        ref13 = O.gemv_tab(g("x13"), g("w13"), g("s13"), g("ids"), g("rw"), 3, False)
        ref2 = O.gemv_tab(g("x2"), g("w2"), g("s2"), g("ids"), g("rw"), 1, True)
        assert O.max_rel_err(o13.float().cpu(), ref13) < TOL
        assert O.max_rel_err(o2.float().cpu(), ref2) < TOL
        # against the reference Triton kernel's own bf16 outputs
        assert O.max_rel_err(o13.float().cpu(), g("o13").float()) < 2 * TOL
        assert O.max_rel_err(o2.float().cpu(), g("o2").float()) < 2 * TOL


def test_reference_unit_test_gemv_replica(pkg, dev):
    """TestInt2Gemv.test_gemv_tab_vs_reference (series-0002:2162-2232) on this implementation."""
    gen = torch.Generator().manual_seed(0)
    e, k13, n13, k2, n2, topk = 8, 256, 200, 128, 256, 3
    for sdtype in (torch.float16, torch.bfloat16):
        q13 = torch.randint(0, 4, (e, k13, n13), generator=gen)
        q2 = torch.randint(0, 4, (e, k2, n2), generator=gen)
        w13 = O.pack_words_along_k(q13.transpose(1, 2)).transpose(1, 2).contiguous()
        w2 = O.pack_words_along_k(q2.transpose(1, 2)).transpose(1, 2).contiguous()
        s13 = (torch.rand(e, k13 // 128, n13, generator=gen) * 0.1 + 0.01).to(sdtype)
        s2 = (torch.rand(e, k2 // 128, n2, generator=gen) * 0.1 + 0.01).to(sdtype)
        ids = torch.randperm(e, generator=gen)[:topk].to(torch.int32)
        x13 = torch.randn(k13, generator=gen).to(torch.bfloat16)
        x2 = torch.randn(topk, k2, generator=gen).to(torch.bfloat16)
        rw = torch.rand(topk, generator=gen) + 0.5
        ref13 = O.gemv_tab(x13[None], w13, s13, ids, rw, topk, False)
        ref2 = O.gemv_tab(x2, w2, s2, ids, rw, 1, True)
        w13d, s13d, w2d, s2d = _cuda(w13, s13, w2, s2, dev=dev)
        wt13, st13, sw13, ss13 = pkg.make_tables(w13d, s13d)
        wt2, st2, sw2, ss2 = pkg.make_tables(w2d, s2d)
        assert (sw13, ss13) == (w13d.stride(1), s13d.stride(1))
        assert wt13.is_cuda and wt13.dtype == torch.int64
        assert int(wt13[3]) == w13d.data_ptr() + 3 * w13d.stride(0) * 4
        assert int(st13[5]) == s13d.data_ptr() + 5 * s13d.stride(0) * 2
        ids_d, rw_d = ids.to(dev), rw.float().to(dev)
        o13 = pkg.moe_gemv_int2_tab(x13[None].to(dev), wt13, st13, ids_d, rw_d, n13, k13, sw13, ss13,
                                    top_k=topk, mul_routed_weight=False, scale_bf16=sdtype == torch.bfloat16)
        o2 = pkg.moe_gemv_int2_tab(x2.to(dev), wt2, st2, ids_d, rw_d, n2, k2, sw2, ss2, top_k=1,
                                   mul_routed_weight=True, scale_bf16=sdtype == torch.bfloat16)
        torch.cuda.synchronize()
        for got, ref in ((o13.float().cpu(), ref13), (o2.float().cpu(), ref2)):
            assert O.norm_rel_err(got, ref) < 1e-2
            assert O.max_rel_err(got, ref) < TOL


@pytest.mark.parametrize("K,N,R,top_k", [(128, 64, 1, 1), (1536, 4096, 8, 1), (4096, 3072, 8, 8), (2048, 1536, 5, 5)])
def test_gemv_with_per_group_zeros(pkg, dev, K, N, R, top_k):
    gen = torch.Generator().manual_seed(K + N + R)
    E = 6
    w = torch.randint(-(2 ** 31), 2 ** 31, (E, K // 16, N), dtype=torch.int32, generator=gen)
    s = (torch.randn(E, K // 128, N, generator=gen).abs() * 0.02).half()
    z = torch.randint(0, 256, (E, K // 128, N // 4), dtype=torch.uint8, generator=gen)
    M = (R + top_k - 1) // top_k
    a = torch.randn(M, K, generator=gen).to(torch.bfloat16)
    ids = torch.randint(0, E, (R,), generator=gen).to(torch.int32)
    rw = torch.rand(R, generator=gen)
    ref = O.gemv_tab(a, w, s, ids, rw, top_k, True, zeros_nc=z)
    wd, sd, zd = _cuda(w, s, z, dev=dev)
    wt, st, sw, ss = pkg.make_tables(wd, sd)
    zt, zs = pkg.make_zero_table(zd)
    out = pkg.moe_gemv_int2_tab(a.to(dev), wt, st, ids.to(dev), rw.to(dev), N, K, sw, ss, top_k=top_k,
                                mul_routed_weight=True, scale_bf16=False, ztab=zt, stride_zg=zs)
    assert O.max_rel_err(out.float().cpu(), ref) < TOL


def test_slots_form_masks_and_matches_tables(pkg, dev):
    gen = torch.Generator().manual_seed(5)
    S, E, K, N = 5, 8, 512, 256
    w = torch.randint(-(2 ** 31), 2 ** 31, (S, K // 16, N), dtype=torch.int32, generator=gen)
    s = (torch.rand(S, K // 128, N, generator=gen) * 0.05).to(torch.bfloat16)
    slots = torch.tensor([3, -1, 0, 4, -1, 1, 2, -1], dtype=torch.int32)
    ids = torch.tensor([0, 1, 2, 3, 4, 5, 6, 7], dtype=torch.int32)
    a = torch.randn(1, K, generator=gen).to(torch.bfloat16)
    wd, sd = _cuda(w, s, dev=dev)
    out = pkg.moe_gemv_int2_slots(a.to(dev), slots.to(dev), wd, sd, ids.to(dev), top_k=8)
    ref = O.gemv_tab(a, w, s, ids, None, 8, False, slots=slots)
    o = out.float().cpu()
    for r in (1, 4, 7):
        assert torch.equal(o[r], torch.zeros(N))                   # slot -1 -> exact zero row
    assert O.max_rel_err(o, ref) < TOL
    # the table form over the same memory gives bit-identical rows
    wt, st, sw, ss = pkg.make_tables(wd, sd)
    ids_slot = torch.tensor([3, 0, 4, 1, 2], dtype=torch.int32)
    o_tab = pkg.moe_gemv_int2_tab(a.to(dev), wt, st, ids_slot.to(dev), None, N, K, sw, ss, top_k=8,
                                  mul_routed_weight=False, scale_bf16=True)
    assert torch.equal(o_tab.cpu(), out[[0, 2, 3, 5, 6]].cpu())


def test_out_of_range_ids_give_zero_rows_and_flag(pkg, dev):
    gen = torch.Generator().manual_seed(9)
    E, K, N = 4, 128, 64
    w = torch.randint(-(2 ** 31), 2 ** 31, (E, K // 16, N), dtype=torch.int32, generator=gen).to(dev)
    s = torch.rand(E, 1, N, generator=gen).half().to(dev)
    wt, st, sw, ss = pkg.make_tables(w, s)
    pkg.last_device_error(dev)
    ids = torch.tensor([1, 7], dtype=torch.int32, device=dev)      # 7 >= E
    out = pkg.moe_gemv_int2_tab(torch.randn(1, K, device=dev).to(torch.bfloat16), wt, st, ids, None, N, K, sw, ss,
                                top_k=2, mul_routed_weight=False, scale_bf16=False)
    assert torch.equal(out[1].cpu(), torch.zeros(N, dtype=torch.bfloat16))
    assert pkg.last_device_error(dev) & 1


def test_to_word_ncontig_gpu_bit_exact(pkg, golden, dev):
    assert torch.equal(pkg.to_word_ncontig(golden["relayout_in"].to(dev)).cpu(), golden["relayout_out"])
    gen = torch.Generator().manual_seed(3)
    for e, n, k in ((3, 64, 256), (2, 640, 2560), (1, 16, 64), (2, 3072, 4096)):
        u8 = torch.randint(0, 256, (e, n, k // 4), dtype=torch.uint8, generator=gen)
        assert torch.equal(pkg.to_word_ncontig(u8.to(dev)).cpu(), O.to_word_ncontig(u8))


def test_gather_rows_tab_bit_exact(pkg, dev):
    gen = torch.Generator().manual_seed(4)
    rows = torch.randint(0, 256, (10, 4096), dtype=torch.uint8, generator=gen).to(dev)
    tab = (torch.arange(10, dtype=torch.int64) * 4096 + rows.data_ptr()).to(dev)
    ids = torch.tensor([7, 0, 7, 3], dtype=torch.int32, device=dev)
    out = torch.empty(4, 4096, dtype=torch.uint8, device=dev)
    pkg._native.call("w2a16_gather_rows_tab", tab.data_ptr(), ids.data_ptr(), 4, out.data_ptr(), 4096,
                     torch.cuda.current_stream().cuda_stream)
    assert torch.equal(out.cpu(), rows[ids.long()].cpu())


def test_gemv_full_size_gate_up(pkg, dev):
    """Config-1 gate_up GEMV: R=8 routed rows, K=4096, N=3072 (the reference's w13 call)."""
    gen = torch.Generator().manual_seed(21)
    E, K, N = 10, 4096, 3072
    w = torch.randint(-(2 ** 31), 2 ** 31, (E, K // 16, N), dtype=torch.int32, generator=gen)
    s = (torch.randn(E, K // 128, N, generator=gen).abs() * 0.02).half()
    a = torch.randn(1, K, generator=gen).to(torch.bfloat16)
    ids = torch.randperm(E, generator=gen)[:8].to(torch.int32)
    wd, sd = _cuda(w, s, dev=dev)
    wt, st, sw, ss = pkg.make_tables(wd, sd)
    out = pkg.moe_gemv_int2_tab(a.to(dev), wt, st, ids.to(dev), None, N, K, sw, ss, top_k=8,
                                mul_routed_weight=False, scale_bf16=False)
    ref = O.gemv_tab(a, w, s, ids, None, 8, False)
    assert O.max_rel_err(out.float().cpu(), ref) < TOL
