"""Expert-parallel decode across the GPUs of one node: experts partitioned 1/N per rank.

Each rank holds, per MoE layer, an arena of its own E/N experts (a contiguous block of expert ids) and a
slot table that maps every other expert to -1. A layer then runs on every rank as

    y_r = moe_decode_layer(x, topk_ids, topk_w, local_arena)   # routed rows of remote experts masked
    y   = all_reduce_sum(y_r)                                    # NCCL over NVLink

so every rank streams only the routed experts it owns and the sum of the partials is the full layer
(each routed expert is owned by exactly one rank). The decode step of BASELINE config 4 stacks L such
layers, each followed by the INT8 dense [H -> H] projection (replicated on every rank), with the step's
activation broadcast from rank 0 at its start. The activation of every later layer is already replicated
by the all-reduce.

The partition and slot-table helpers are pure host logic (tested on CPU with gloo ranks); the layer and
the INT8 GEMV are the package's CUDA kernels, so the step itself needs CUDA devices.
"""
from __future__ import annotations

import json
import os
import time
from dataclasses import dataclass
from datetime import timedelta
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

__all__ = ["expert_range", "local_slot_table", "shard_arena", "ep_moe_layer", "EPDecodeStep", "bench_main"]


def expert_range(num_experts: int, world: int, rank: int) -> Tuple[int, int]:
    """Experts [lo, hi) owned by `rank`: contiguous blocks, sizes differing by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    return rank * num_experts // world, (rank + 1) * num_experts // world


def local_slot_table(num_experts: int, world: int, rank: int, device=None) -> torch.Tensor:
    """int32 [E]: slot of each locally owned expert in this rank's arena (0 .. hi-lo-1), -1 elsewhere."""
    lo, hi = expert_range(num_experts, world, rank)
    slots = torch.full((num_experts,), -1, dtype=torch.int32)
    slots[lo:hi] = torch.arange(hi - lo, dtype=torch.int32)
    return slots if device is None else slots.to(device)


def shard_arena(codes13, scales13, codes2, scales2, zeros13, zeros2, world: int, rank: int):
    """Slice stacked per-expert tensors ([E, ...], expert-major) to this rank's block; returns the six
    tensors (contiguous) and the local slot table. Works on CPU or CUDA tensors."""
    E = codes13.shape[0]
    lo, hi = expert_range(E, world, rank)
    cut = lambda t: None if t is None else t[lo:hi].contiguous()
    return (cut(codes13), cut(scales13), cut(codes2), cut(scales2), cut(zeros13), cut(zeros2),
            local_slot_table(E, world, rank, codes13.device))


class PeerAllReduce:
    """The library's one-shot all-reduce (w2a16_allreduce_peers_bf16) over NVLink peer memory for small
    bf16 vectors (up to n_max elements). Peer-visible buffers come from torch symmetric memory (set up once,
    collectively); every call is one kernel launch with no host involvement, so it can sit in a CUDA graph.
    Sums run in rank order in fp32 and are bit-identical on every rank."""

    def __init__(self, n_max: int, device: torch.device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        from . import _native
        self._native = _native
        self.group = group if group is not None else dist.group.WORLD
        self.n_max = n_max
        world = dist.get_world_size(self.group)
        self.flag_off = ((n_max * 4 * world + 255) // 256) * 256
        self.buf = symm_mem.empty(self.flag_off + 4 * max(world, 64), dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        self.rank, self.world = self.handle.rank, self.handle.world_size
        self.peers = torch.tensor([int(a) for a in self.handle.buffer_ptrs], dtype=torch.int64, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def check(self) -> int:
        """Read and clear the kernel's device error word (bit 1: a flag wait gave up, i.e. a rank did not
        arrive within the wait limit). Synchronises with the device: call it between steps, outside graph
        capture. Raises RuntimeError when a bit is set, so a stalled peer does not go unnoticed."""
        v = int(self.err.item())
        if v:
            self.err.zero_()
            raise RuntimeError(f"peer all-reduce: device error word {v:#x} (bit 1 = a rank's flag never arrived)")
        return v

    def __call__(self, y: torch.Tensor) -> torch.Tensor:
        if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.numel() > self.n_max:
            raise ValueError("PeerAllReduce takes a contiguous bf16 tensor of at most n_max elements")
        out = torch.empty_like(y)
        self._native.call("w2a16_allreduce_peers_bf16", y.data_ptr(), out.data_ptr(), y.numel(), self.n_max,
                          self.peers.data_ptr(), self.flag_off, self.rank, self.world, self.epoch.data_ptr(),
                          self.err.data_ptr(), torch.cuda.current_stream(y.device).cuda_stream)
        return out


def ep_moe_layer(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, local_arena,
                 routed_scaling_factor: float = 1.0, group=None, allreduce: Optional[PeerAllReduce] = None
                 ) -> torch.Tensor:
    """One expert-parallel MoE layer: this rank's partial over its own experts, summed over the group by
    `allreduce` (the peer-memory kernel) or, when None, by NCCL."""
    from .moe_layer import moe_decode_layer
    y = moe_decode_layer(x, topk_ids, topk_weights, local_arena, routed_scaling_factor)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        if allreduce is not None:
            return allreduce(y)
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y


@dataclass
class EPDecodeStep:
    """L stacked (MoE layer -> INT8 dense projection) blocks on this rank."""
    arenas: List[object]               # ExpertArena per layer (local experts only)
    dense_q: List[torch.Tensor]        # int32 [H/4, H] per layer
    dense_s: List[torch.Tensor]        # f16 [1, H] per layer
    group: Optional[object] = None
    allreduce: Optional[PeerAllReduce] = None

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x bf16 [M, H] (rank 0's copy is broadcast), ids int32 [L, M, k], w f32 [L, M, k] -> bf16 [M, H]."""
        from .int8_gemv import int8_gemv
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.broadcast(x, src=0, group=self.group)
        for l, arena in enumerate(self.arenas):
            y = ep_moe_layer(x, ids[l], w[l], arena, group=self.group, allreduce=self.allreduce)
            x = int8_gemv(y, self.dense_q[l], self.dense_s[l])
        return x


# ----------------------------------------------------------------------------- config 4 benchmark
def _layer_bytes(H: int, I: int, k: int, M: int) -> int:
    """Algorithmic weight bytes of one routed expert set (codes + fp16 scales + zero points)."""
    per = (H // 16) * 2 * I * 4 + (H // 128) * 2 * I * 2 + (H // 128) * (2 * I // 4) \
        + (I // 16) * H * 4 + (I // 128) * H * 2 + (I // 128) * (H // 4)
    return per * k * M


def bench_main(args) -> None:
    """Config 4 under torchrun: L=48 stacked layers, E=256 experts partitioned over the ranks, top-8,
    M=1, each layer followed by the INT8 [4096 -> 4096] projection. Device-timed per rank with CUDA events
    over CUDA-graph replays of whole steps; the max over ranks is reported."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        _bench_ep(args, rank, world, dev)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _bench_ep(args, rank: int, world: int, dev: torch.device) -> None:
    from . import synth
    from .moe_layer import ExpertArena, moe_decode_layer
    import bench as B
    L, E, H, I, k, M = 48, 256, 4096, 1536, 8, 1
    lo, hi = expert_range(E, world, rank)
    slots = local_slot_table(E, world, rank, dev)
    t0 = time.time()
    arenas = []
    for l in range(L):
        a = synth.make_arena(hi - lo, H, I, seed=7919 * l + lo, zeros=True, scale_dtype=torch.float16, device=dev)
        arenas.append(ExpertArena(a.codes13, a.scales13, a.codes2, a.scales2, a.zeros13, a.zeros2, slots))
    dense = [synth.make_int8_dense(H, H, seed=104729 + l, device=dev) for l in range(L)]
    ar = PeerAllReduce(M * H, dev)
    step = EPDecodeStep(arenas, [d[0] for d in dense], [d[1] for d in dense], allreduce=ar)
    P = 8                                          # routings / activations cycled by the timed graph
    ids_all, w_all = B.routing_pool(P * L, E, k, window=4, seed=0)
    ids_d = ids_all.reshape(P, L, M, k).to(dev)
    w_d = w_all.reshape(P, L, M, k).to(dev)
    x_d = synth.make_activation(P * M, H, seed=0, device=dev).reshape(P, M, H)
    x_in = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    setup_s = time.time() - t0

    # correctness of one expert-parallel layer: GPU all-reduced output vs the all-reduced fp32 oracle
    # partials of every rank's own experts
    import oracle as O
    y0 = ep_moe_layer(x_d[0].clone(), ids_d[0, 0], w_d[0, 0], arenas[0])
    ref = O.moe_layer_from_arena(arenas[0], x_d[0], ids_d[0, 0], w_d[0, 0]).to(dev)
    dist.all_reduce(ref)
    err = O.max_rel_err(y0.float().cpu(), ref.cpu())
    # the peer-memory all-reduce against NCCL's on the same partial
    part = moe_decode_layer(x_d[0].clone(), ids_d[0, 0], w_d[0, 0], arenas[0])
    mine = ar(part)
    nccl = part.float().clone()
    dist.all_reduce(nccl)
    ar_err = O.max_rel_err(mine.float().cpu(), nccl.cpu())
    ar_flag = int(ar.err.item())
    ar_us = {}
    for name, fn in (("peer", lambda t: ar(t)), ("nccl", lambda t: dist.all_reduce(t))):
        bufs = [part.clone() for _ in range(48)]
        for t in bufs[:4]:
            fn(t)
        torch.cuda.synchronize()
        ga = torch.cuda.CUDAGraph()
        sa = torch.cuda.Stream()
        sa.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(sa):
            with torch.cuda.graph(ga, stream=sa):
                for t in bufs:
                    fn(t)
        torch.cuda.current_stream().wait_stream(sa)
        ga.replay()
        torch.cuda.synchronize()
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(5):
            ga.replay()
        a1.record()
        torch.cuda.synchronize()
        del ga
        tm = torch.tensor([a0.elapsed_time(a1) * 1e3 / (5 * 48)], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ar_us[name] = round(float(tm.item()), 2)

    def run(i):
        x_in.copy_(x_d[i % P])
        return step(x_in, ids_d[i % P], w_d[i % P])

    for i in range(max(args.warmup, 3)):
        run(i)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        run(0)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            for i in range(P):
                run(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    reps = max(1, -(-args.steps // P))
    steps = reps * P
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with B.ClockSampler(dev.index or 0) as clk:
        dist.barrier()
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(reps):
            g.replay()
        ev1.record()
        torch.cuda.synchronize()
        dist.barrier()
    del g                                          # no graph holding NCCL work outlives the timed region
    torch.cuda.synchronize()
    ms = torch.tensor([ev0.elapsed_time(ev1)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    us_step = float(ms.item()) * 1e3 / steps

    # e2e: pinned host activation and routing copied in, the step's output copied out, every step
    xh = x_d.cpu().pin_memory()
    ih = ids_d.cpu().pin_memory()
    wh = w_d.cpu().pin_memory()
    out_h = torch.empty(M, H, dtype=torch.bfloat16).pin_memory()
    ids_buf, w_buf = torch.empty_like(ids_d[0]), torch.empty_like(w_d[0])
    K_e = min(steps, 16)
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K_e):
        x_in.copy_(xh[i % P], non_blocking=True)
        ids_buf.copy_(ih[i % P], non_blocking=True)
        w_buf.copy_(wh[i % P], non_blocking=True)
        out = step(x_in, ids_buf, w_buf)
        out_h.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    me = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(me, op=dist.ReduceOp.MAX)
    e2e_us = float(me.item()) * 1e3 / K_e
    h2d = x_in.numel() * 2 + ids_buf.numel() * 4 + w_buf.numel() * 4
    d2h = out_h.numel() * 2

    moe_bytes = _layer_bytes(H, I, k, M)
    dense_bytes = (H // 4) * H * 4 + H * 2
    step_bytes = L * (moe_bytes + dense_bytes)     # algorithmic bytes of the step, dense counted once
    gbs = step_bytes / (us_step * 1e-6) / 1e9
    peak, peak_kind = B.peaks()
    per_gpu = gbs / world
    if rank == 0:
        line = {
            "metric": B.METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(us_step / 1e3, 6), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u2xbf16->fp32 (int32 exact group sums); int8 dense",
            "data": "synthetic (seeded; BASELINE config 4 distributions)",
            "config": {"workload": f"config4: decode step, 48 x (MoE layer E=256 top-8 H=4096 I=1536 W2A16 g128 "
                                   f"-> INT8 dense 4096x4096), experts {E // world} per GPU",
                       "global_batch": M, "seq_len": 1, "parallelism": f"ep{world} (peer-memory all-reduce per layer)",
                       "l2": f"inputs larger than L2 ({(hi - lo) * L} local experts, {L * 16} MB dense per GPU)"},
            "us_per_step": round(us_step, 2), "us_per_layer": round(us_step / L, 3),
            "bytes_per_step": step_bytes,
            "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(per_gpu / peak, 4), "traffic": None,
                         "kernel": "whole step per GPU (fused MoE layer + peer all-reduce + INT8 GEMV), algorithmic bytes / N",
                         "peak_kind": peak_kind},
            "e2e": {"value": round(step_bytes / (e2e_us * 1e-6) / 1e9, 1), "unit": "GB/s",
                    "us_per_step": round(e2e_us, 1), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "how": "eager EPDecodeStep calls; pinned host activation + routing in, output out"},
            "gpu_launches": steps * L * 2,
            "clocks": clk.summary(),
            "check_max_rel_err": err,
            "allreduce": {"impl": "w2a16_allreduce_peers_bf16 (one-shot over NVLink peer memory)",
                          "max_rel_err_vs_nccl_fp32": ar_err, "device_error_word": ar_flag,
                          "us_per_call_graph": ar_us},
            "setup_s": round(setup_s, 1),
        }
        print(json.dumps(line), flush=True)
