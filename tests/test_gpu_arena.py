"""Native arenas on the GPU: rows written through a view survive growth; the elastic layer arena grows and shrinks
under a CUDA graph captured once, with the slot table rewritten in place, and the replayed layer always matches
the oracle for the current residency (gemv/expert_elastic.py:198-252 is the behaviour checked)."""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def test_row_arena_real_driver(pkg, dev):
    a = pkg.arena.RowArena(256 << 10, 24, device_id=dev.index or 0, chunk_bytes=2 << 20, name="t")
    assert a.ensure_rows(8) > 0 and a.backed_rows >= 8
    v = a.view(a.backed_rows, (64 << 10,), torch.int32)
    v[:8].copy_(torch.arange(8 * (64 << 10), dtype=torch.int32, device=dev).view(8, -1))
    base = a.base
    assert a.ensure_rows(24) > 0 and a.base == base                    # the rows did not move
    v = a.view(24, (64 << 10,), torch.int32)
    assert torch.equal(v[:8].flatten().cpu(), torch.arange(8 * (64 << 10), dtype=torch.int32))
    v[20].fill_(7)
    torch.cuda.synchronize()
    assert a.shrink_rows(8) > 0 and a.backed_rows >= 8 and a.backed_rows < 24
    assert torch.equal(a.view(8, (64 << 10,), torch.int32)[3].cpu(), torch.arange(3 * (64 << 10), 4 * (64 << 10),
                                                                                  dtype=torch.int32))
    a.close()


def test_elastic_arena_under_a_captured_graph(pkg, dev):
    E, H, I, k = 16, 1024, 512, 4
    g = torch.Generator().manual_seed(61)
    host = {}
    for e in range(E):
        host[e] = {"codes13": torch.randint(-(2 ** 31), 2 ** 31, (H // 16, 2 * I), dtype=torch.int32, generator=g),
                   "scales13": (torch.randn(H // 128, 2 * I, generator=g).abs() * 0.02).half(),
                   "zeros13": torch.randint(0, 256, (H // 128, 2 * I // 4), dtype=torch.uint8, generator=g),
                   "codes2": torch.randint(-(2 ** 31), 2 ** 31, (I // 16, H), dtype=torch.int32, generator=g),
                   "scales2": (torch.randn(I // 128, H, generator=g).abs() * 0.02).half(),
                   "zeros2": torch.randint(0, 256, (I // 128, H // 4), dtype=torch.uint8, generator=g)}
        host[e] = {n: t.pin_memory() for n, t in host[e].items()}
    ea = pkg.arena.ElasticExpertArena(E, H, I, max_slots=16, device=dev, chunk_bytes=2 << 20)
    order = torch.randperm(E, generator=g).tolist()
    ea.resize(order, 4, host.__getitem__)
    x = pkg.synth.make_activation(2, H, seed=61, device=dev, gen_device="cpu")
    ids, w = pkg.synth.route_softmax(2, E, k, seed=61, device=dev, gen_device="cpu")
    y = torch.empty(2, H, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        pkg.moe_decode_layer(x, ids, w, ea.arena, out=y)
        with torch.cuda.graph(graph, stream=s):
            pkg.moe_decode_layer(x, ids, w, ea.arena, out=y)
    torch.cuda.current_stream().wait_stream(s)
    for S in (4, 12, 16, 3, 9):
        ea.resize(order, S, host.__getitem__)
        before = ea.backed_bytes()
        graph.replay()
        torch.cuda.synchronize()
        assert pkg.last_device_error(dev) == 0
        ref = O.moe_layer_by_expert(ea.arena, x, ids, w)
        assert O.max_rel_err(y.float().cpu(), ref) < TOL, S
        assert int((ea.slots >= 0).sum()) == S and before == ea.backed_bytes()
    del graph
    ea.close()
