"""Worker of tests/test_gpu_multi_exchange.py (one process per GPU under torch.distributed.run): a 2-rank stack of
expert-parallel layers with the exchange folded into the kernels against (layer, all-reduce) per layer, bit for
bit, and its first layer against the oracle of the whole (unsharded) layer. Prints "OK <rank>" on success."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__ as graft  # noqa: E402
import oracle as O  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    pkg = graft.load_package()
    ep = pkg.expert_parallel
    E, H, I, k, M, L = 32, 1024, 512, 8, 1, 4
    full = [pkg.synth.make_arena(E, H, I, seed=60 + l, zeros=True, device=dev, gen_device="cpu") for l in range(L)]
    lo, hi = ep.expert_range(E, world, rank)
    slots = ep.local_slot_table(E, world, rank, dev)
    arenas = [pkg.ExpertArena(a.codes13[lo:hi].contiguous(), a.scales13[lo:hi].contiguous(), a.codes2[lo:hi].contiguous(),
                              a.scales2[lo:hi].contiguous(), a.zeros13[lo:hi].contiguous(), a.zeros2[lo:hi].contiguous(),
                              slots) for a in full]
    ids, w = zip(*[pkg.synth.route_softmax(M, E, k, seed=5 + l, device=dev, gen_device="cpu") for l in range(L)])
    ids, w = torch.stack(ids), torch.stack(w)
    x = pkg.synth.make_activation(M, H, seed=9, device=dev, gen_device="cpu")
    ch = ep.PeerAllReduce(M * H, dev, spin_limit=1 << 20)
    ref = x
    for l in range(L):
        ref = ch(pkg.moe_decode_layer(ref, ids[l], w[l], arenas[l]))
    got = ep.ep_stack_step(ch, x, ids, w, arenas)
    y0 = ch(pkg.moe_decode_layer(x, ids[0], w[0], arenas[0]))
    torch.cuda.synchronize()
    ok = torch.equal(got, ref) and int(ch.err.item()) == 0
    err = O.max_rel_err(y0.float().cpu(), O.moe_layer_from_arena(full[0], x, ids[0], w[0]))
    ok = ok and err < 1e-2
    t = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    del ch
    dist.barrier()
    dist.destroy_process_group()
    print(("OK " if int(t.item()) == 1 else "FAIL ") + str(rank), "rel_err", err, flush=True)
    return 0 if int(t.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
