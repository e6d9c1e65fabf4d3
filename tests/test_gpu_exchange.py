"""The exchange folded into the kernels (w2a16_moe_decode_layer_slots_ep, w2a16_int8_gemv_from_peers) on one GPU,
over a world-1 channel (the rank's own buffer, no process group): a chain of layers that push their partials and
sum them into the next layer's activation gives, bit for bit, what (layer, all-reduce) per layer gives, the INT8
projection reading from the channel equals the projection of the layer's output, and the channel's epoch
advances once per push. The failure path makes a word wait run out (a call whose words nothing writes) with a short wait limit: bit 1 of the error word, the call completes, the context stays
usable. No fault, trap or unbounded wait is involved."""
import time

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

E, H, I, K = 32, 1024, 512, 8


def _arenas(pkg, dev, n):
    return [pkg.synth.make_arena(E, H, I, seed=40 + l, zeros=True, device=dev, gen_device=dev) for l in range(n)]


def _routing(pkg, dev, M, n, seed=7):
    ids, w = [], []
    for l in range(n):
        i, ww = pkg.synth.route_softmax(M, E, K, seed=seed + l, device=dev, gen_device=dev)
        ids.append(i)
        w.append(ww)
    return torch.stack(ids), torch.stack(w)


@pytest.mark.parametrize("M", [1, 2])
def test_pushed_chain_equals_layer_allreduce_chain(pkg, dev, M):
    L = 4
    arenas = _arenas(pkg, dev, L)
    ids, w = _routing(pkg, dev, M, L)
    x = pkg.synth.make_activation(M, H, seed=3, device=dev)
    ep = pkg.expert_parallel
    ch = ep.PeerAllReduce(M * H, dev, local=True)
    ref = x
    for l in range(L):
        ref = ch(pkg.moe_decode_layer(ref, ids[l], w[l], arenas[l]))
    torch.cuda.synchronize()
    e0 = int(ch.epoch.item())
    assert e0 == L
    got = ep.ep_stack_step(ch, x, ids, w, arenas)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    assert int(ch.epoch.item()) == e0 + L           # L - 1 pushes and the closing all-reduce
    assert int(ch.err.item()) == 0
    # the layer's own pieces: push, then a plain-output layer reading the sum
    ch.layer(x, ids[0], w[0], arenas[0], y_to_peers=True)
    y1 = ch.layer(None, ids[1], w[1], arenas[1], x_from_peers=True)
    y1_ref = pkg.moe_decode_layer(pkg.moe_decode_layer(x, ids[0], w[0], arenas[0]), ids[1], w[1], arenas[1])
    torch.cuda.synchronize()
    assert torch.equal(y1, y1_ref)


def test_int8_from_peers_equals_projection_of_layer(pkg, dev):
    M = 1
    arena = _arenas(pkg, dev, 1)[0]
    ids, w = _routing(pkg, dev, M, 1)
    x = pkg.synth.make_activation(M, H, seed=5, device=dev)
    q, s = pkg.synth.make_int8_dense(H, H, seed=11, device=dev)
    ch = pkg.expert_parallel.PeerAllReduce(M * H, dev, local=True)
    ch.layer(x, ids[0], w[0], arena, y_to_peers=True)
    z = ch.int8(q, s, M)
    z_ref = pkg.int8_gemv(pkg.moe_decode_layer(x, ids[0], w[0], arena), q, s)
    torch.cuda.synchronize()
    assert torch.equal(z, z_ref)
    assert int(ch.err.item()) == 0


def test_exchange_wait_gives_up_when_no_flag_arrives(pkg, dev):
    M = 1
    arena = _arenas(pkg, dev, 1)[0]
    ids, w = _routing(pkg, dev, M, 1)
    q, s = pkg.synth.make_int8_dense(H, H, seed=12, device=dev)
    ch = pkg.expert_parallel.PeerAllReduce(M * H, dev, spin_limit=2000, local=True)
    ch.epoch.fill_(5)                               # call 5: nothing ever raises its flag
    t0 = time.perf_counter()
    ch.layer(None, ids[0], w[0], arena, x_from_peers=True)
    torch.cuda.synchronize()
    assert int(ch.err.item()) & 2                    # the layer's wait gave up and said so
    ch.err.zero_()
    ch.int8(q, s, M)
    torch.cuda.synchronize()
    assert int(ch.err.item()) & 2                    # and the projection's
    assert time.perf_counter() - t0 < 10.0
    with pytest.raises(RuntimeError):
        ch.check()
    # the context is usable: a plain layer afterwards matches the oracle
    x = pkg.synth.make_activation(M, H, seed=6, device=dev)
    y = pkg.moe_decode_layer(x, ids[0], w[0], arena)
    err = O.max_rel_err(y.float().cpu(), O.moe_layer_from_arena(arena, x, ids[0], w[0]))
    assert err < 1e-2
