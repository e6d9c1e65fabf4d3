"""Run the decode MoE layer a fixed number of times on one GPU -- the command that profiling captures use.

    python qwen3.8-flash-next-24gb-sglang_b200/microbench/layer_case.py --experts 256 --calls 6

Builds a resident arena of `--experts` experts at config-1 shapes (H=4096, I=1536, W2A16 g128 with zero
points, fp16 scales), draws a fresh top-8 routing for every call (no expert repeats within 4 calls), runs
the calls through the public layer entry point and checks the last one against the CPU oracle. With
`--experts 32` the arena (160 MB) still exceeds L2 while keeping a full ncu capture small.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--calls", type=int, default=6)
    ap.add_argument("--M", type=int, default=1)
    args = ap.parse_args()
    import __graft_entry__ as graft
    import oracle as O
    from bench import routing_pool

    pkg = graft.load_package()
    dev = torch.device("cuda", 0)
    E, H, I, k, M = args.experts, 4096, 1536, 8, args.M
    arena = pkg.synth.make_arena(E, H, I, seed=0, zeros=True, scale_dtype=torch.float16, device=dev)
    ids_pool, w_pool = routing_pool(args.calls * M, E, k, window=min(4, max(1, E // (2 * k))), seed=0)
    x = pkg.synth.make_activation(args.calls * M, H, seed=0, device=dev)
    ids = ids_pool.to(dev)
    ws = w_pool.to(dev)
    y = None
    for c in range(args.calls):
        sl = slice(c * M, (c + 1) * M)
        y = pkg.moe_decode_layer(x[sl], ids[sl], ws[sl], arena)
    torch.cuda.synchronize()
    sl = slice((args.calls - 1) * M, args.calls * M)
    err = O.max_rel_err(y.float().cpu(), O.moe_layer_from_arena(arena, x[sl], ids[sl], ws[sl]))
    print(f"layer_case: E={E} M={M} calls={args.calls} max_rel_err={err:.2e}")
    return 0 if err < 1e-2 else 1


if __name__ == "__main__":
    raise SystemExit(main())
