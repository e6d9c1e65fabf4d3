"""Host-side behaviour of the drop-in Python API that needs no GPU."""
import pytest
import torch


def test_gemv_rejects_bad_block(pkg):
    """series-0002:2234-2248: K=64 with the default block_k=128 raises AssertionError before any work."""
    with pytest.raises(AssertionError):
        pkg.moe_gemv_int2_tab(torch.zeros(1, 64, dtype=torch.bfloat16), None, None,
                              torch.zeros(1, dtype=torch.int32), None, 8, 64, 8, 8, top_k=1,
                              mul_routed_weight=False)


def test_cpu_tensors_are_rejected(pkg):
    """There is no CPU path: CPU inputs raise instead of silently computing elsewhere."""
    with pytest.raises(ValueError):
        pkg.moe_gemv_int2_tab(torch.zeros(1, 128, dtype=torch.bfloat16), None, None,
                              torch.zeros(1, dtype=torch.int32), None, 8, 128, 8, 8, top_k=1,
                              mul_routed_weight=False)
    with pytest.raises(ValueError):
        pkg.to_word_ncontig(torch.zeros(1, 8, 4, dtype=torch.int32))
    if not torch.cuda.is_available():
        # a host tensor is relayouted by the CUDA kernel over unified addressing; without a device it raises
        with pytest.raises(RuntimeError):
            pkg.to_word_ncontig(torch.zeros(1, 8, 4, dtype=torch.uint8))
    with pytest.raises(ValueError):
        pkg.int8_gemv(torch.zeros(1, 128, dtype=torch.bfloat16), torch.zeros(32, 8, dtype=torch.int32),
                      torch.zeros(1, 8, dtype=torch.float16))


def test_missing_library_raises(pkg, monkeypatch, tmp_path):
    """Without the built library every op raises at its first call; nothing computes elsewhere."""
    nat = pkg._native
    monkeypatch.setattr(nat, "_lib", None)
    monkeypatch.setattr(nat, "LIB_PATH", str(tmp_path / "absent" / "libw2a16_moe.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        nat.lib()
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        pkg.version()


def test_synth_distributions(pkg):
    s = pkg.synth
    pop = s.zipf_popularity(256, 1.1, seed=0)
    assert abs(float(pop.sum()) - 1.0) < 1e-5
    slots = s.resident_slots(pop, 184, seed=0)
    assert int((slots >= 0).sum()) == 184
    assert sorted(slots[slots >= 0].tolist()) == list(range(184))
    ids, w = s.route_zipf(64, 256, 8, pop, seed=0, device="cpu")
    assert ids.shape == (64, 8) and all(len(set(r.tolist())) == 8 for r in ids)
    assert torch.allclose(w.sum(-1), torch.ones(64))
    ids, w = s.route_softmax(4, 256, 8, seed=0, device="cpu")
    assert torch.allclose(w.sum(-1), torch.ones(4)) and ids.dtype == torch.int32
    qw, sc = s.make_int8_dense(256, 64, seed=0, device="cpu")
    import oracle as O
    q = O.int8_unpack(qw) - 128
    assert int(q.min()) >= -127 and int(q.max()) <= 127 and sc.shape == (1, 64)


def test_gemv_gate_mirrors_the_reference(pkg):
    """MoeWNA16Method.apply's gate (patches/ncontig_gemv.py:249-253): word layout, 2-bit, at most 16 tokens,
    SGLANG_MOE_GEMV unset or "1"."""
    from types import SimpleNamespace
    word = SimpleNamespace(_b_n_contig=True)
    byte = SimpleNamespace()
    g = pkg.use_gemv
    assert g(word, 1, env={}) and g(word, 16, env={}) and g(word, 16, env={"SGLANG_MOE_GEMV": "1"})
    assert not g(word, 17, env={})
    assert not g(word, 1, env={"SGLANG_MOE_GEMV": "0"})
    assert not g(word, 1, weight_bits=4, env={})
    assert not g(byte, 1, env={})
    assert pkg.moe_method.GEMV_MAX_TOKENS == 16


def test_relayout_switch_leaves_layer_untouched(pkg, monkeypatch):
    """SGLANG_MOE_NCONTIG=0 (and non-2-bit layers) skip the relayout, as the reference does
    (patches/ncontig_gemv.py:177-180); nothing runs, so no GPU is needed."""
    from types import SimpleNamespace
    t = torch.zeros(2, 8, 4, dtype=torch.uint8)
    layer = SimpleNamespace(w13_qweight=t, w2_qweight=t, w13_scales=t, w2_scales=t)
    monkeypatch.setenv("SGLANG_MOE_NCONTIG", "0")
    pkg.MoeWNA16Method().process_weights_after_loading(layer)
    assert layer.w13_qweight is t and not getattr(layer, "_b_n_contig", False)
    monkeypatch.setenv("SGLANG_MOE_NCONTIG", "1")
    pkg.MoeWNA16Method(weight_bits=4).process_weights_after_loading(layer)
    assert layer.w13_qweight is t and not getattr(layer, "_b_n_contig", False)
