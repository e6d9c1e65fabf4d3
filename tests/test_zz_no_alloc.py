"""The decode-layer entry point that allocates nothing (w2a16_moe_decode_layer_slots_noalloc).

It serves callers that cannot allocate device memory — a host that reaches the layer while its stream
is being captured into a CUDA graph, or a serving process whose device memory is all reserved by its
own pool — and therefore cannot pass a workspace. Its scratch is a fixed array inside the library.
The test calls it through the C ABI twice in a row and compares each result with the regular entry
point (which takes a workspace), at the tolerance the layer tests use. This file is collected last so
that a failure here leaves every other test already run; it passes alone in a fresh process as well.
"""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _call_noalloc(pkg, x, ids, w, arena, y, M=None, H=None, I=None):
    lib = pkg._native.lib()
    esz = arena.scales13.element_size()
    M = x.shape[0] if M is None else M
    H = arena.H if H is None else H
    I = arena.I if I is None else I
    return lib.w2a16_moe_decode_layer_slots_noalloc(
        x.data_ptr(), M, H, I, ids.shape[1], ids.data_ptr(), w.data_ptr(), arena.slots.data_ptr(),
        arena.E, arena.S, arena.codes13.data_ptr(), arena.codes13.stride(0) * 4, arena.scales13.data_ptr(),
        arena.scales13.stride(0) * esz, arena.zeros13.data_ptr(), arena.zeros13.stride(0),
        arena.codes2.data_ptr(), arena.codes2.stride(0) * 4, arena.scales2.data_ptr(),
        arena.scales2.stride(0) * esz, arena.zeros2.data_ptr(), arena.zeros2.stride(0),
        int(arena.scale_bf16), 1.0, y.data_ptr(), None, torch.cuda.current_stream().cuda_stream)


def test_noalloc_entry_matches_workspace_entry(pkg, dev):
    E, H, I, M, k = 32, 2048, 768, 2, 8
    slots = torch.randperm(E, generator=torch.Generator().manual_seed(3)).to(torch.int32)
    slots[5] = -1                                         # one expert not resident
    arena = pkg.synth.make_arena(E, H, I, seed=11, zeros=True, device=dev, gen_device="cpu", slots=slots)
    x = pkg.synth.make_activation(M, H, seed=11, device=dev, gen_device="cpu")
    ids, w = pkg.synth.route_softmax(M, E, k, seed=11, device=dev, gen_device="cpu")
    ref = pkg.moe_decode_layer(x, ids, w, arena)          # the existing entry point, with a workspace
    for _ in range(2):                                    # two calls in a row share the fixed scratch
        y = torch.full_like(ref, float("nan"))
        assert _call_noalloc(pkg, x, ids, w, arena, y) == 0
        torch.cuda.synchronize()
        assert O.max_rel_err(y.float().cpu(), ref.float().cpu()) <= TOL
        assert torch.isfinite(y.float()).all()


@pytest.mark.parametrize("M", [16, 64])
def test_noalloc_entry_full_size_token_batches(pkg, dev, M):
    """Config-3 shapes (H=4096, I=1536, E=256, top-8) at 16 and 64 tokens, two calls in a row: the no-alloc
    entry takes the per-token path below 64 tokens like the regular entry (its choice follows the token
    count, not the size of its array), and at 64 tokens, where the batched path's buffers do not fit the
    array, the per-token path too; both agree with the regular entry within the layer tolerance."""
    E, H, I, k = 256, 4096, 1536, 8
    arena = pkg.synth.make_arena(E, H, I, seed=21, zeros=True, device=dev, gen_device=dev)
    x = pkg.synth.make_activation(M, H, seed=21, device=dev, gen_device=dev)
    ids, w = pkg.synth.route_softmax(M, E, k, seed=21, device=dev, gen_device=dev, uniform_logits=True)
    ref = pkg.moe_decode_layer(x, ids, w, arena)
    for _ in range(2):
        y = torch.full_like(ref, float("nan"))
        assert _call_noalloc(pkg, x, ids, w, arena, y) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all()
        assert O.max_rel_err(y.float().cpu(), ref.float().cpu()) <= TOL


def test_noalloc_entry_rejects_oversized_layers(pkg, dev):
    arena = pkg.synth.make_arena(4, 256, 512, seed=12, zeros=True, device=dev, gen_device="cpu")
    x = torch.zeros(1, 256, dtype=torch.bfloat16, device=dev)
    ids = torch.zeros(1, 8, dtype=torch.int32, device=dev)
    w = torch.zeros(1, 8, dtype=torch.float32, device=dev)
    y = torch.empty(1, 256, dtype=torch.bfloat16, device=dev)
    # the smallest token count whose workspace exceeds the 4 MiB scratch is refused before any launch or
    # memory access
    lib = pkg._native.lib()
    M = 1
    while lib.w2a16_moe_layer_workspace_bytes(M, 4096, 1536, 8) <= 4 << 20:
        M += 1
    assert _call_noalloc(pkg, x, ids, w, arena, y, M=M, H=4096, I=1536) == 5
