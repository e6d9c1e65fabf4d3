"""The peer all-reduce kernel on one GPU: a call with world 1, and the failure path -- a rank whose flag never
arrives. With world 2 and both peer addresses pointing at this GPU's own buffer, "rank 1" never raises its flag:
the kernel must give up after the test's short wait limit, set bit 1 of the error word, finish, and leave the
context usable (the next call on the stream runs normally). No fault, trap or unbounded wait is involved."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _flag_off(n, world):
    return ((n * 4 * world + 255) // 256) * 256


def _buffer(n, world, dev):
    """A peer buffer of the documented layout: 2 parity slots x world rows x n bf16, then `world` uint32 flags at
    flag_off (zero)."""
    return torch.zeros(_flag_off(n, world) + 4 * 64, dtype=torch.uint8, device=dev)


def _call(pkg, dev, world, rank, n, buf, peers, epoch, err, spin_limit, x):
    out = torch.empty_like(x)
    flag_off = _flag_off(n, world)
    assert buf.numel() >= flag_off + 4 * world
    st = pkg._native.lib().w2a16_allreduce_peers_bf16(
        x.data_ptr(), out.data_ptr(), n, n, peers.data_ptr(), flag_off, rank, world, epoch.data_ptr(), err.data_ptr(),
        spin_limit, torch.cuda.current_stream(dev).cuda_stream)
    assert st == 0
    return out


def test_allreduce_world_one_is_identity(pkg, dev):
    n = 4096
    buf = _buffer(n, 1, dev)
    peers = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    x = torch.randn(n, device=dev).to(torch.bfloat16)
    for _ in range(3):
        out = _call(pkg, dev, 1, 0, n, buf, peers, epoch, err, 0, x)
        torch.cuda.synchronize()
        assert torch.equal(out, x) and int(err.item()) == 0
    assert int(epoch.item()) == 3


def test_allreduce_wait_gives_up_when_a_rank_never_arrives(pkg, dev):
    n = 4096
    buf = _buffer(n, 2, dev)
    peers = torch.tensor([buf.data_ptr(), buf.data_ptr()], dtype=torch.int64, device=dev)   # both "ranks" here
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    x = torch.randn(n, device=dev).to(torch.bfloat16)
    t0 = time.perf_counter()
    _call(pkg, dev, 2, 0, n, buf, peers, epoch, err, 2000, x)          # rank 1's flag never comes
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(err.item()) & 2                                           # the wait gave up and said so
    assert int(epoch.item()) == 1                                        # and the call completed
    # the context is usable: a world-1 call on the same stream runs and returns the identity
    err.zero_()
    buf1 = _buffer(n, 1, dev)
    peers1 = torch.tensor([buf1.data_ptr()], dtype=torch.int64, device=dev)
    ep1 = torch.zeros(1, dtype=torch.int32, device=dev)
    out = _call(pkg, dev, 1, 0, n, buf1, peers1, ep1, err, 0, x)
    torch.cuda.synchronize()
    assert torch.equal(out, x) and int(err.item()) == 0
