"""Expert-parallel host logic on CPU: the 1/N expert partition, the local slot
tables, and that the sum over gloo ranks of each rank's partial layer (fp32 oracle over its own experts,
remote experts masked through slot -1) equals the full layer. The GPU step itself runs in bench.py
under torchrun; these tests need no GPU."""
import os
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O


@pytest.mark.parametrize("E,world", [(256, 1), (256, 2), (256, 8), (64, 3), (10, 4)])
def test_partition_covers_every_expert_once(pkg, E, world):
    owner = torch.full((E,), -1)
    for r in range(world):
        lo, hi = pkg.expert_parallel.expert_range(E, world, r)
        assert hi - lo in (E // world, E // world + 1)
        assert (owner[lo:hi] == -1).all()
        owner[lo:hi] = r
    assert (owner >= 0).all()


def test_local_slot_tables(pkg):
    E, world = 256, 4
    seen = torch.zeros(E, dtype=torch.int32)
    for r in range(world):
        slots = pkg.expert_parallel.local_slot_table(E, world, r)
        lo, hi = pkg.expert_parallel.expert_range(E, world, r)
        assert slots.dtype == torch.int32
        assert torch.equal(slots[lo:hi], torch.arange(hi - lo, dtype=torch.int32))
        assert (slots[:lo] == -1).all() and (slots[hi:] == -1).all()
        seen += (slots >= 0).int()
    assert (seen == 1).all()


def _cpu_model(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    words = lambda shape: torch.randint(-2**31, 2**31, shape, dtype=torch.int64, generator=g).to(torch.int32)
    scales = lambda shape: (torch.randn(shape, generator=g).abs() * 0.02).to(torch.float16)
    return (words((E, H // 16, 2 * I)), scales((E, H // 128, 2 * I)), words((E, I // 16, H)),
            scales((E, I // 128, H)), torch.randint(0, 256, (E, H // 128, 2 * I // 4), dtype=torch.uint8, generator=g),
            torch.randint(0, 256, (E, I // 128, H // 4), dtype=torch.uint8, generator=g))


def _rank_main(rank, world, port, E, H, I, k, M, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import __graft_entry__ as graft
        pkg = graft.load_package()
        c13, s13, c2, s2, z13, z2 = _cpu_model(E, H, I, seed=5)
        parts = pkg.expert_parallel.shard_arena(c13, s13, c2, s2, z13, z2, world, rank)
        local = types.SimpleNamespace(codes13=parts[0], scales13=parts[1], codes2=parts[2], scales2=parts[3],
                                      zeros13=parts[4], zeros2=parts[5], slots=parts[6])
        g = torch.Generator().manual_seed(6)
        x = torch.randn(M, H, generator=g).to(torch.bfloat16)
        ids, w = O.route_topk(torch.randn(M, E, generator=g), k)
        y = O.moe_layer_from_arena(local, x, ids.to(torch.int32), w)
        dist.all_reduce(y)
        if rank == 0:
            full = types.SimpleNamespace(codes13=c13, scales13=s13, codes2=c2, scales2=s2, zeros13=z13, zeros2=z2,
                                         slots=torch.arange(E, dtype=torch.int32))
            ref = O.moe_layer_from_arena(full, x, ids.to(torch.int32), w)
            out_q.put(float((y - ref).abs().max() / ref.abs().max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sum_of_rank_partials_is_the_full_layer(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, 16, 256, 256, 4, 2, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    rel = q.get(timeout=5)
    assert rel < 1e-5, rel
