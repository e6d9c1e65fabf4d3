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

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

__all__ = ["expert_range", "local_slot_table", "shard_arena", "PeerAllReduce", "ep_moe_layer", "EPDecodeStep"]


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

    def __init__(self, n_max: int, device: torch.device, group=None, spin_limit: int = 0):
        import torch.distributed._symmetric_memory as symm_mem
        from . import _native
        self._native = _native
        self.group = group if group is not None else dist.group.WORLD
        self.n_max = n_max
        self.spin_limit = int(spin_limit)      # polls before a flag wait gives up (0: the library's default)
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
                          self.err.data_ptr(), self.spin_limit, torch.cuda.current_stream(y.device).cuda_stream)
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
    """L stacked (MoE layer -> INT8 dense projection) blocks on this rank. With ``check_errors`` every call
    first reads (and clears) the peer all-reduce's device error word -- a host synchronisation, so it is skipped
    while a CUDA graph is being captured -- and raises when a flag wait gave up in an earlier step."""
    arenas: List[object]               # ExpertArena per layer (local experts only)
    dense_q: List[torch.Tensor]        # int32 [H/4, H] per layer
    dense_s: List[torch.Tensor]        # f16 [1, H] per layer
    group: Optional[object] = None
    allreduce: Optional[PeerAllReduce] = None
    check_errors: bool = False

    def check(self) -> None:
        """Raise RuntimeError when the peer all-reduce reported a wait that gave up (step boundaries only)."""
        if self.allreduce is not None:
            self.allreduce.check()

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x bf16 [M, H] (rank 0's copy is broadcast), ids int32 [L, M, k], w f32 [L, M, k] -> bf16 [M, H]."""
        from .int8_gemv import int8_gemv
        if self.check_errors and not torch.cuda.is_current_stream_capturing():
            self.check()
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.broadcast(x, src=0, group=self.group)
        for l, arena in enumerate(self.arenas):
            y = ep_moe_layer(x, ids[l], w[l], arena, group=self.group, allreduce=self.allreduce)
            x = int8_gemv(y, self.dense_q[l], self.dense_s[l])
        return x
