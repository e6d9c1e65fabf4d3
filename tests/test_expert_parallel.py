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


@pytest.mark.parametrize("world,k,M", [(2, 4, 2), (4, 1, 1)])
def test_sum_of_rank_partials_is_the_full_layer(world, k, M):
    """(4, 1, 1): one routed expert, so three of the four ranks hold no routed expert and contribute zeros."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000) + 7 * world
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, 16, 256, 256, k, M, q)) for r in range(world)]
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


# ----------------------------------------------------------------------------- peer all-reduce protocol model
class _ArModel:
    """The one-shot peer all-reduce's protocol (csrc/w2a16_allreduce.cu) as a step-by-step model: call e of a
    rank writes its row into parity slot e & 1 of every rank's buffer, raises its flag to e on every rank, waits
    until each of its own flags reached e, sums the rows of its own slot, and stores e as its epoch. `signed`
    selects the kernel's wait (flag - e >= 0 as a signed distance) or an equality wait (flag == e)."""

    def __init__(self, world, signed):
        self.world, self.signed = world, signed
        self.rows = [[[None] * world for _ in range(2)] for _ in range(world)]   # [rank][slot][row]
        self.flags = [[0] * world for _ in range(world)]
        self.epoch = [0] * world
        self.results = [[] for _ in range(world)]
        self.max_polls = [0] * world

    def rank(self, r, calls, poll_limit):
        for e in range(1, calls + 1):
            for q in range(self.world):                     # push this call's row into every rank's slot e & 1
                self.rows[q][e & 1][r] = (e, r)
                yield
            for q in range(self.world):                     # raise the flag on every rank
                self.flags[q][r] = e
                yield
            for q in range(self.world):                     # wait for every rank's row (bounded)
                polls = 0
                while not ((self.flags[r][q] - e >= 0) if self.signed else (self.flags[r][q] == e)):
                    polls += 1
                    if polls > poll_limit:
                        raise TimeoutError(f"rank {r} call {e}: flag of rank {q} is {self.flags[r][q]}")
                    yield
                self.max_polls[r] = max(self.max_polls[r], polls)
            self.results[r].append(tuple(self.rows[r][e & 1]))   # the rows this rank sums
            self.epoch[r] = e
            yield


def _run_model(world, calls, seed, signed, order=None, poll_limit=10_000):
    import random
    m = _ArModel(world, signed)
    gens = {r: m.rank(r, calls, poll_limit) for r in range(world)}
    rnd = random.Random(seed)
    sched = iter(order) if order is not None else None
    while gens:
        r = next(sched) if sched is not None else rnd.choice(sorted(gens))
        if r not in gens:
            continue
        try:
            next(gens[r])
        except StopIteration:
            del gens[r]
    return m


@pytest.mark.parametrize("world", [2, 4, 8])
def test_allreduce_protocol_sums_the_right_rows(world):
    """Under random interleavings every rank sums, for every call e, exactly the rows all ranks wrote for call e
    (a slot is never overwritten while a rank still reads it), and no wait gives up."""
    for seed in range(20):
        m = _run_model(world, 12, seed, signed=True)
        for r in range(world):
            assert m.results[r] == [tuple((e, q) for q in range(world)) for e in range(1, 13)]
            assert m.epoch[r] == 12


def test_allreduce_equality_wait_misses_a_flag_that_moved_on():
    """A fast rank can finish call e and raise its flag to e + 1 before a slow rank polls it. An equality wait
    then never sees e and gives up although the row is in place; the signed-distance wait the kernel uses
    accepts e + 1 and sums the right rows."""
    # rank 1 runs call 1 to its end and pushes call 2's rows and flags; only then does rank 0 start polling
    order = [1] * 2 + [0] * 2 + [0] * 2 + [1] * 30 + [0] * 60
    with pytest.raises(TimeoutError):
        _run_model(2, 2, 0, signed=False, order=order + [0] * 100, poll_limit=50)
    m = _run_model(2, 2, 0, signed=True, order=order + [0, 1] * 200, poll_limit=50)
    assert m.results[0] == [((1, 0), (1, 1)), ((2, 0), (2, 1))]
