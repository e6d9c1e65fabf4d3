"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py) and against the reference's known-answer checks."""
import torch

import oracle as O

# the reference's GEMV bar (series-0002:2231-2232) and bf16 output rounding
TOL_GEMV = 1e-2


def test_relayout_bit_exact(golden):
    assert torch.equal(O.to_word_ncontig(golden["relayout_in"]), golden["relayout_out"])


def test_word_and_byte_packing_bit_exact(golden):
    q = golden["zp_words_vals"]
    assert torch.equal(O.pack_words_along_k(q), golden["zp_words"])
    assert torch.equal(O.pack_2bit_along_last(q), golden["zp_bytes"])


def test_to_word_ncontig_known_answer():
    """series-0002:1989-2010: bit-exact, every value at bits 2*(k%16) of word k//16, invertible."""
    gen = torch.Generator().manual_seed(7)
    for e, n, k in ((3, 64, 256), (2, 640, 2560), (1, 16, 64)):
        q = torch.randint(0, 4, (e, n, k), generator=gen)
        byte = O.pack_2bit_along_last(q)
        word = O.to_word_ncontig(byte)
        assert word.dtype == torch.int32 and word.shape == (e, k // 16, n) and word.is_contiguous()
        assert torch.equal(word, O.pack_words_along_k(q).transpose(1, 2).contiguous())
        for kk in (0, 1, 15, 16, 17, k - 1):
            assert torch.equal((word[:, kk // 16, :] >> (2 * (kk % 16))) & 3, q[:, :, kk].to(torch.int32))
        back = word.view(torch.uint8).view(e, k // 16, n, 4).permute(0, 2, 1, 3).reshape(e, n, k // 4)
        assert torch.equal(back, byte)


def test_unpack_known_answer():
    """series-0002:2013-2081 / tools/test_group_layout.py:20-38: unpack of words is bit-exact."""
    gen = torch.Generator().manual_seed(7)
    for k, n, gs in ((2560, 640, 128), (640, 2560, 128), (256, 64, 64)):
        vals = torch.randint(0, 4, (k, n), dtype=torch.int32, generator=gen)
        sc = (torch.rand(k // gs, n, generator=gen) * 0.02 + 0.001).float()
        words = O.pack_words_along_k(vals.T.contiguous()).T.contiguous()     # [K/16, N]
        assert torch.equal(O.unpack_words(words), vals)
        ref = (vals.float() - 2) * sc.repeat_interleave(gs, dim=0)
        assert torch.equal(O.dequant(words, sc, group=gs), ref)


def test_gemv_matches_reference_triton(golden):
    for s in ("f16", "bf16"):
        g = lambda k: golden[f"tab_{s}_{k}"]
        o13 = O.gemv_tab(g("x13"), g("w13"), g("s13"), g("ids"), g("rw"), 3, False)
        o2 = O.gemv_tab(g("x2"), g("w2"), g("s2"), g("ids"), g("rw"), 1, True)
        assert O.max_rel_err(g("o13").float(), o13) < TOL_GEMV
        assert O.max_rel_err(g("o2").float(), o2) < TOL_GEMV
        assert O.norm_rel_err(g("o13").float(), o13) < 5e-3


def test_byte_gemv_matches_reference_triton(golden):
    ob = O.gemv_byte_tab(golden["byte_x"], golden["byte_q"], golden["byte_s"], golden["byte_ids"])
    assert O.max_rel_err(golden["byte_out"], ob) < 1e-5


def test_per_group_zero_points_match_reference_helpers(golden):
    """make_int2_experts(has_zp=True) (series-0002:1936-1954): loader bytes + qzeros -> word layout ->
    oracle dequant reproduces the reference's bf16 dequantized weights exactly."""
    for w in ("w1", "w2"):
        words = O.to_word_ncontig(golden[f"zp_{w}_q"])
        sc = golden[f"zp_{w}_s"].transpose(1, 2).contiguous()
        zn = O.zeros_to_ncontig(golden[f"zp_{w}_zp"])
        deq = O.dequant(words, sc, zn)
        assert torch.equal(deq.to(torch.bfloat16), golden[f"zp_{w}_ref"].transpose(1, 2))


def test_package_zero_point_relayout_matches_oracle(pkg, golden):
    """The package's loader conversion of qzeros (zeros_to_ncontig, a host-side transpose the GEMV form is
    made with) equals the oracle's on the reference's golden per-group zero points, byte for byte."""
    for w in ("w1", "w2"):
        qz = golden[f"zp_{w}_zp"]
        got = pkg.zeros_to_ncontig(qz)
        assert got.dtype == torch.uint8 and got.is_contiguous()
        assert torch.equal(got, O.zeros_to_ncontig(qz))


def test_moe_layer_matches_reference_torch_moe(golden):
    """torch_moe (series-0002:1957-1973, bf16 math, softmax without renormalisation) vs the fp32 oracle."""
    topk = int(golden["zp_topk"])
    words13 = O.to_word_ncontig(golden["zp_w1_q"]); s13 = golden["zp_w1_s"].transpose(1, 2).contiguous()
    words2 = O.to_word_ncontig(golden["zp_w2_q"]); s2 = golden["zp_w2_s"].transpose(1, 2).contiguous()
    z13 = O.zeros_to_ncontig(golden["zp_w1_zp"]); z2 = O.zeros_to_ncontig(golden["zp_w2_zp"])
    ids, w = O.route_topk(golden["zp_score"].float(), topk, renormalize=False)
    y = O.moe_layer(golden["zp_a"], words13, s13, words2, s2, ids, w, z13=z13, z2=z2)
    assert O.max_rel_err(golden["zp_moe"].float(), y) < 2e-2      # TOL atol 1e-3 / rtol 2e-2 (:1916)


def test_int8_formula_matches_reference(golden):
    """unpack_int8_gptq (scripts/requant_int8.py:53-63) == oracle unpack/dequant; GEMV consistent."""
    qw, qz, sc = golden["int8_qw"], golden["int8_qz"], golden["int8_sc"]
    assert (qz == 0x7F7F7F7F).all()                        # symmetric: stored zero - 1 = 127
    q = O.int8_unpack(qw).float()
    W = (q - 128.0) * sc.float().repeat_interleave(128, dim=0)        # [K, N]
    assert torch.equal(W.T.contiguous(), golden["int8_deq"])
    x = torch.randn(2, qw.shape[0] * 4, generator=torch.Generator().manual_seed(3))
    y = O.int8_gemv(x, qw, sc)
    assert O.max_rel_err(y, x @ golden["int8_deq"].T) < 1e-5


def test_int8_pack_roundtrip():
    gen = torch.Generator().manual_seed(11)
    q = torch.randint(0, 256, (256, 64), generator=gen)
    assert torch.equal(O.int8_unpack(O.int8_pack(q)), q.to(torch.int32))


def test_zero_point_relayout_roundtrip():
    gen = torch.Generator().manual_seed(2)
    zp = torch.randint(0, 4, (3, 64, 4), generator=gen)           # [E, N, K/g]
    qz = O.pack_zeros(zp)                                         # [E, N/4, K/g]
    nc = O.zeros_to_ncontig(qz)                                   # [E, K/g, N/4]
    assert torch.equal(O.unpack_zeros_nc(nc), zp.transpose(1, 2).to(torch.int32))


def test_slot_masking_semantics():
    gen = torch.Generator().manual_seed(4)
    E, K, N = 4, 128, 32
    w = torch.randint(-(2 ** 31), 2 ** 31, (E, K // 16, N), dtype=torch.int32, generator=gen)
    s = torch.rand(E, K // 128, N, generator=gen).half()
    a = torch.randn(1, K, generator=gen).to(torch.bfloat16)
    ids = torch.tensor([0, 3, 1], dtype=torch.int32)
    slots = torch.tensor([2, -1, 0, 1], dtype=torch.int32)
    o = O.gemv_tab(a, w, s, ids, None, 3, False, slots=slots)
    assert torch.equal(o[2], torch.zeros(N))                     # expert 1 not resident
    assert torch.allclose(o[0], O.gemv_tab(a, w, s, torch.tensor([2], dtype=torch.int32), None, 1, False)[0])


def test_expert_order_oracle_matches_token_order():
    """moe_layer_by_expert (each expert dequantised once, for whole token batches) computes the same
    layer as the token-order loop moe_layer_routed_only, masked and out-of-arena slots included."""
    from types import SimpleNamespace
    gen = torch.Generator().manual_seed(9)
    E, S, H, I, M, k = 8, 6, 256, 128, 5, 3
    rw = lambda *sh: torch.randint(-(2 ** 31), 2 ** 31, sh, dtype=torch.int32, generator=gen)
    ar = SimpleNamespace(codes13=rw(S, H // 16, 2 * I), scales13=(torch.rand(S, H // 128, 2 * I, generator=gen) * 0.02).half(),
                         zeros13=torch.randint(0, 256, (S, H // 128, 2 * I // 4), dtype=torch.uint8, generator=gen),
                         codes2=rw(S, I // 16, H), scales2=(torch.rand(S, I // 128, H, generator=gen) * 0.02).half(),
                         zeros2=torch.randint(0, 256, (S, I // 128, H // 4), dtype=torch.uint8, generator=gen),
                         slots=torch.tensor([0, 1, -1, 2, 3, 4, 5, 99], dtype=torch.int32))
    x = torch.randn(M, H, generator=gen).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=gen)[:k] for _ in range(M)]).to(torch.int32)
    w = torch.softmax(torch.randn(M, k, generator=gen), -1)
    experts = {}
    for e in range(E):
        sl = int(ar.slots[e])
        if 0 <= sl < S:
            experts[e] = (ar.codes13[sl], ar.scales13[sl], ar.zeros13[sl], ar.codes2[sl], ar.scales2[sl],
                          ar.zeros2[sl])
    a = O.moe_layer_routed_only(x, experts, ids, w, 1.5)
    b = O.moe_layer_by_expert(ar, x, ids, w, 1.5)
    assert torch.allclose(a, b, rtol=1e-5, atol=1e-6)


def test_oracle_layer_with_no_resident_routed_expert_is_zero():
    """A rank of an expert-parallel step may hold none of the routed experts: its partial is zero."""
    from types import SimpleNamespace
    H, I, M, k = 256, 128, 2, 2
    ar = SimpleNamespace(codes13=torch.zeros(1, H // 16, 2 * I, dtype=torch.int32),
                         scales13=torch.ones(1, H // 128, 2 * I, dtype=torch.float16), zeros13=None,
                         codes2=torch.zeros(1, I // 16, H, dtype=torch.int32),
                         scales2=torch.ones(1, I // 128, H, dtype=torch.float16), zeros2=None,
                         slots=torch.tensor([-1, -1, -1, 0], dtype=torch.int32))
    x = torch.randn(M, H, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    ids = torch.tensor([[0, 1], [2, 1]], dtype=torch.int32)
    w = torch.full((M, k), 0.5)
    y = O.moe_layer_from_arena(ar, x, ids, w, 2.0)
    assert y.shape == (M, H) and torch.equal(y, torch.zeros(M, H))
