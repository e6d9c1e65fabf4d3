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

:class:`PeerAllReduce` is also an exchange channel that folds the all-reduce into the kernels: a layer can push
its partial straight into every rank's buffer as its units finish (``y_to_peers``), and the next layer -- or the
INT8 projection -- sums the ranks' rows while it converts its activation (``x_from_peers``). A step is then one
launch per layer (and per projection) with no separate all-reduce.

The partition and slot-table helpers are pure host logic (tested on CPU with gloo ranks); the layer and
the INT8 GEMV are the package's CUDA kernels, so the step itself needs CUDA devices.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

__all__ = ["expert_range", "local_slot_table", "shard_arena", "PeerAllReduce", "ep_moe_layer", "EPDecodeStep",
           "ep_stack_step"]


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
    bf16 vectors (up to n_max elements), and the exchange channel (w2a16_exchange) of the fused expert-parallel
    calls :meth:`layer` and :meth:`int8`, which share its buffers, flags and epoch word. Peer-visible buffers come
    from torch symmetric memory (set up once, collectively); every call is one kernel launch with no host
    involvement, so it can sit in a CUDA graph. Sums run in rank order in fp32 and are bit-identical on every
    rank. ``local=True`` makes a world-1 channel over plain device memory (no process group; one GPU)."""

    def __init__(self, n_max: int, device: torch.device, group=None, spin_limit: int = 0, local: bool = False):
        from . import _native
        self._native = _native
        self.n_max = n_max
        self.spin_limit = int(spin_limit)      # polls before a flag wait gives up (0: the library's default)
        self.device = torch.device(device)
        # buffer: the all-reduce's 2 x world x n_max bf16 slots, its flags at flag_off, then the tagged exchange
        # words (2 x world x n_max / 2 of 8 bytes) at tag_off
        if local:
            self.group, world, self.rank, self.world = None, 1, 0, 1
        else:
            self.group = group if group is not None else dist.group.WORLD
            world = dist.get_world_size(self.group)
        self.flag_off = ((n_max * 4 * world + 255) // 256) * 256
        self.tag_off = self.flag_off + 4 * max(world, 64)
        nbytes = self.tag_off + 8 * world * n_max
        if local:
            self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
            self.peers = torch.tensor([self.buf.data_ptr()], dtype=torch.int64, device=device)
        else:
            import torch.distributed._symmetric_memory as symm_mem
            self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
            self.buf.zero_()
            self.handle = symm_mem.rendezvous(self.buf, self.group)
            self.rank, self.world = self.handle.rank, self.handle.world_size
            self.peers = torch.tensor([int(a) for a in self.handle.buffer_ptrs], dtype=torch.int64, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.exchange = _native.Exchange(self.peers.data_ptr(), self.tag_off, n_max, self.rank, self.world,
                                         self.epoch.data_ptr(), self.spin_limit)
        torch.cuda.synchronize(device)
        if not local:
            dist.barrier(group=self.group)

    def check(self) -> int:
        """Read and clear the kernels' device error word (bit 1: a flag wait gave up, i.e. a rank did not
        arrive within the wait limit). Synchronises with the device: call it between steps, outside graph
        capture. Raises RuntimeError when a bit is set, so a stalled peer does not go unnoticed."""
        v = int(self.err.item())
        if v:
            self.err.zero_()
            raise RuntimeError(f"peer exchange: device error word {v:#x} (bit 1 = a rank's flag never arrived)")
        return v

    def __call__(self, y: torch.Tensor) -> torch.Tensor:
        if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.numel() > self.n_max:
            raise ValueError("PeerAllReduce takes a contiguous bf16 tensor of at most n_max elements")
        out = torch.empty_like(y)
        self._native.call("w2a16_allreduce_peers_bf16", y.data_ptr(), out.data_ptr(), y.numel(), self.n_max,
                          self.peers.data_ptr(), self.flag_off, self.rank, self.world, self.epoch.data_ptr(),
                          self.err.data_ptr(), self.spin_limit, torch.cuda.current_stream(y.device).cuda_stream)
        return out

    def layer(self, x: Optional[torch.Tensor], topk_ids: torch.Tensor, topk_weights: torch.Tensor, arena,
              routed_scaling_factor: float = 1.0, x_from_peers: bool = False, y_to_peers: bool = False,
              out: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """This rank's MoE layer over its local arena (w2a16_moe_decode_layer_slots_ep). ``x_from_peers``: the
        activation is the sum of the ranks' rows of the channel's current call (x is ignored and may be None);
        ``y_to_peers``: the partial goes to every rank as this rank's row of the next call and nothing is
        returned; otherwise the partial (bf16 [M, H]) is returned (in ``out`` when given)."""
        from .moe_layer import _err_word, _p, _stream, _workspace_bytes, layer_workspace
        ids = topk_ids.to(torch.int32).contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        M, top_k = ids.shape
        H = arena.codes2.shape[2]
        I = arena.codes13.shape[2] // 2
        if M * H > self.n_max:
            raise ValueError(f"M * H = {M * H} exceeds the channel's n_max {self.n_max}")
        if not x_from_peers and (x is None or x.dtype != torch.bfloat16 or tuple(x.shape) != (M, H)
                                 or x.device != self.device):
            raise ValueError("x must be a bf16 [M, H] tensor on the channel's device unless x_from_peers")
        for t in (ids, w, arena.slots, arena.codes13, arena.scales13, arena.codes2, arena.scales2):
            if t.device != self.device:
                raise ValueError("routing and arena tensors must be on the channel's device")
        xx = None if x_from_peers else x.contiguous()
        y = None
        if not y_to_peers:
            y = torch.empty((M, H), dtype=torch.bfloat16, device=self.device) if out is None else out
        nbytes = _workspace_bytes(M, H, I, top_k, 0)
        ws = layer_workspace(self.device, nbytes)
        esz = arena.scales13.element_size()
        self._native.call(
            "w2a16_moe_decode_layer_slots_ep", _p(xx), M, H, I, top_k, ids.data_ptr(), w.data_ptr(),
            arena.slots.data_ptr(), arena.slots.numel(), arena.codes13.shape[0],
            arena.codes13.data_ptr(), arena.codes13.stride(0) * 4, arena.scales13.data_ptr(),
            arena.scales13.stride(0) * esz, _p(arena.zeros13), 0 if arena.zeros13 is None else arena.zeros13.stride(0),
            arena.codes2.data_ptr(), arena.codes2.stride(0) * 4, arena.scales2.data_ptr(), arena.scales2.stride(0) * esz,
            _p(arena.zeros2), 0 if arena.zeros2 is None else arena.zeros2.stride(0),
            int(arena.scales13.dtype == torch.bfloat16), float(routed_scaling_factor), _p(y), ws.data_ptr(), nbytes,
            int(bool(x_from_peers)), int(bool(y_to_peers)), ctypes.byref(self.exchange), self.err.data_ptr(),
            _stream(self.device))
        return y

    def int8(self, qweight: torch.Tensor, scales: torch.Tensor, M: int, zero: int = 128,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The INT8 projection of the sum of the ranks' rows of the channel's current call (w2a16_int8_gemv_from_peers):
        rows of K = 4 * qweight.shape[0] values -> bf16 [M, N]."""
        K, N = qweight.shape[0] * 4, qweight.shape[1]
        if qweight.device != self.device or scales.device != self.device or not qweight.is_contiguous():
            raise ValueError("qweight (contiguous) and scales must be on the channel's device")
        if M * K > self.n_max:
            raise ValueError(f"M * K = {M * K} exceeds the channel's n_max {self.n_max}")
        group = K if scales.shape[0] == 1 else K // scales.shape[0]
        y = torch.empty((M, N), dtype=torch.bfloat16, device=self.device) if out is None else out
        self._native.call("w2a16_int8_gemv_from_peers", ctypes.byref(self.exchange), qweight.data_ptr(),
                          scales.data_ptr(), group, int(zero), M, K, N, y.data_ptr(), y.stride(0), self.err.data_ptr(),
                          torch.cuda.current_stream(self.device).cuda_stream)
        return y


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
    fused: bool = False                # with ``allreduce``: layers push their partials, the projections sum them

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
        if self.fused and self.allreduce is not None:
            M = x.shape[0]
            for l, arena in enumerate(self.arenas):
                self.allreduce.layer(x, ids[l], w[l], arena, y_to_peers=True)
                x = self.allreduce.int8(self.dense_q[l], self.dense_s[l], M)
            return x
        for l, arena in enumerate(self.arenas):
            y = ep_moe_layer(x, ids[l], w[l], arena, group=self.group, allreduce=self.allreduce)
            x = int8_gemv(y, self.dense_q[l], self.dense_s[l])
        return x


def ep_stack_step(channel: PeerAllReduce, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, arenas: List[object],
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """L stacked expert-parallel MoE layers, each layer's input the previous layer's output, with the exchange
    folded into the layers: layer 0 reads x and pushes its partial, layers 1 .. L-1 sum the ranks' partials while
    they convert their activation and push theirs (the last one returns its partial instead), and one all-reduce
    ends the step. Same result, bit for bit, as (layer, all-reduce) per layer. x bf16 [M, H] (replicated),
    ids int32 [L, M, k], w f32 [L, M, k]."""
    L = len(arenas)
    if L == 1:
        return channel(channel.layer(x, ids[0], w[0], arenas[0], out=out))
    channel.layer(x, ids[0], w[0], arenas[0], y_to_peers=True)
    for l in range(1, L - 1):
        channel.layer(None, ids[l], w[l], arenas[l], x_from_peers=True, y_to_peers=True)
    y = channel.layer(None, ids[L - 1], w[L - 1], arenas[L - 1], x_from_peers=True, out=out)
    return channel(y)
