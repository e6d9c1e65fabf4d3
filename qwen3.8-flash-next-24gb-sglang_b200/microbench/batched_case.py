"""Time the decode MoE layer at several token counts (config 3) on one GPU, batched path against per-token path.

    python qwen3.8-flash-next-24gb-sglang_b200/microbench/batched_case.py --M 4 16 64 --calls 40

Config-3 shapes (H=4096, I=1536, E=256 resident, top-8, W2A16 g128 with zero points, fp16 scales) and a fresh
uniform-random routing for every call. Each path runs `--calls` layers captured in one CUDA graph; the time per
layer is the replay's CUDA-event time divided by the calls. Bytes per layer count every distinct routed expert
once (what a path that streams each expert once must read). The per-token path is the same slot-form entry
point given a workspace below the batched path's size (w2a16_moe_layer_workspace_bytes), the batched path
the size w2a16_moe_layer_workspace_bytes_batched reports at 64 tokens, which selects it from 16 tokens. The last call of each path is checked
against the CPU oracle.
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
    ap.add_argument("--M", type=int, nargs="+", default=[4, 16, 64])
    ap.add_argument("--calls", type=int, default=40)
    args = ap.parse_args()
    import __graft_entry__ as graft
    import oracle as O

    pkg = graft.load_package()
    nat = pkg._native
    dev = torch.device("cuda", 0)
    E, H, I, k = 256, 4096, 1536, 8
    arena = pkg.synth.make_arena(E, H, I, seed=0, zeros=True, scale_dtype=torch.float16, device=dev, gen_device=dev)
    per_expert = arena.bytes_per_expert()
    rc = 0
    for M in args.M:
        P = args.calls
        x = pkg.synth.make_activation(P * M, H, seed=M, device=dev, gen_device=dev).reshape(P, M, H)
        ids, w = pkg.synth.route_softmax(P * M, E, k, seed=M, device=dev, gen_device=dev, uniform_logits=True)
        ids = ids.reshape(P, M, k).contiguous(); w = w.reshape(P, M, k).contiguous()
        distinct = sum(int(torch.unique(ids[c]).numel()) for c in range(P)) / P
        small = int(nat.lib().w2a16_moe_layer_workspace_bytes(M, H, I, k))
        big = int(nat.lib().w2a16_moe_layer_workspace_bytes_batched(max(M, 64), H, I, k))   # batched from 16 tokens
        res = {}
        for name, nbytes in (("batched", big), ("per-token", small)):
            if name == "batched" and M < 16:
                continue                                   # below 16 tokens there is one path
            ws = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=dev)
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            y = torch.empty(P, M, H, dtype=torch.bfloat16, device=dev)

            def call(c, s):
                nat.call("w2a16_moe_decode_layer_slots", x[c].data_ptr(), M, H, I, k, ids[c].data_ptr(),
                         w[c].data_ptr(), arena.slots.data_ptr(), E, arena.codes13.data_ptr(),
                         arena.codes13.stride(0) * 4, arena.scales13.data_ptr(), arena.scales13.stride(0) * 2,
                         arena.zeros13.data_ptr(), arena.zeros13.stride(0), arena.codes2.data_ptr(),
                         arena.codes2.stride(0) * 4, arena.scales2.data_ptr(), arena.scales2.stride(0) * 2,
                         arena.zeros2.data_ptr(), arena.zeros2.stride(0), 0, 1.0, y[c].data_ptr(), ws.data_ptr(),
                         nbytes, err.data_ptr(), s)

            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                for c in range(min(P, 3)):
                    call(c, s.cuda_stream)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for c in range(P):
                        call(c, s.cuda_stream)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            g.replay(); torch.cuda.synchronize()
            times = []
            for _ in range(3):
                e0.record(); g.replay(); e1.record(); torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1) * 1e3 / P)
            us = sorted(times)[1]
            c = P - 1
            rel = O.max_rel_err(y[c].float().cpu(), O.moe_layer_from_arena(arena, x[c], ids[c], w[c]))
            res[name] = us
            ok = rel < 1e-2 and int(err.item()) == 0
            rc |= 0 if ok else 1
            print(f"M={M:3d} {name:9s}: {us:8.1f} us/layer  distinct experts {distinct:6.1f}  "
                  f"{distinct * per_expert / us / 1e3:7.1f} GB/s  max_rel_err {rel:.2e}  err {int(err.item())}")
        if len(res) == 2:
            print(f"M={M:3d} per-token / batched = {res['per-token'] / res['batched']:.2f}x")
    return rc


if __name__ == "__main__":
    raise SystemExit(main())
