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
        pkg.to_word_ncontig(torch.zeros(1, 8, 4, dtype=torch.uint8))
    with pytest.raises(ValueError):
        pkg.int8_gemv(torch.zeros(1, 128, dtype=torch.bfloat16), torch.zeros(32, 8, dtype=torch.int32),
                      torch.zeros(1, 8, dtype=torch.float16))


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
