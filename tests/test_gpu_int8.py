"""GPU parity of the INT8 dense projection GEMV against the CPU oracle (scripts/requant_int8.py
dequant rule). Bar: max relative error <= 1e-2 on bf16 outputs."""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (3, 1024, 512), (5, 384, 128)])
def test_int8_per_channel(pkg, dev, M, K, N):
    qw, sc = pkg.synth.make_int8_dense(K, N, seed=M, device=dev, gen_device="cpu")
    x = pkg.synth.make_activation(M, K, seed=M, device=dev, gen_device="cpu")
    y = pkg.int8_gemv(x, qw, sc)
    ref = O.int8_gemv(x.cpu(), qw.cpu(), sc.cpu())
    assert O.max_rel_err(y.float().cpu(), ref) < 1e-2


@pytest.mark.parametrize("M,K,N", [(9, 1024, 512), (1, 8192, 256), (2, 1024, 132)])
def test_int8_cluster_kernel_shapes(pkg, dev, M, K, N):
    """Shapes the column-slice kernel does not take -- more than 8 tokens, K above 4096, N not a multiple of 8 --
    run the cluster split-K kernel: the same parity bar, with per-channel and with g128 scales."""
    qw, sc = pkg.synth.make_int8_dense(K, N, seed=K + N, device=dev, gen_device="cpu")
    x = pkg.synth.make_activation(M, K, seed=M + 1, device=dev, gen_device="cpu")
    y = pkg.int8_gemv(x, qw, sc)
    assert O.max_rel_err(y.float().cpu(), O.int8_gemv(x.cpu(), qw.cpu(), sc.cpu())) < 1e-2
    sg = (sc.float().repeat(K // 128, 1) * torch.linspace(0.5, 1.5, K // 128, device=dev)[:, None]).to(torch.float16)
    y = pkg.int8_gemv(x, qw, sg)
    assert O.max_rel_err(y.float().cpu(), O.int8_gemv(x.cpu(), qw.cpu(), sg.cpu())) < 1e-2


def test_int8_grouped_scales_and_repeat(pkg, golden, dev):
    """The reference packing with g128 scales (pack_int8_gptq), called twice (ticket counters reset)."""
    qw, sc = golden["int8_qw"].to(dev), golden["int8_sc"].to(dev)
    x = torch.randn(2, qw.shape[0] * 4, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    ref = O.int8_gemv(x, golden["int8_qw"], golden["int8_sc"])
    for _ in range(2):
        y = pkg.int8_gemv(x.to(dev), qw, sc)
        assert O.max_rel_err(y.float().cpu(), ref) < 1e-2


def _int8_torch_fp32(x, qw, sc, zero=128):
    """Plain PyTorch fp32 reference of the INT8 projection on the GPU, 16,384 columns at a time: byte i of int32
    word kw is weight row 4 kw + i, (q - zero) * scale of its 128-row group."""
    K, N = 4 * qw.shape[0], qw.shape[1]
    group = K // sc.shape[0]
    out = torch.empty(x.shape[0], N, dtype=torch.float32, device=x.device)
    xf = x.float()
    for n0 in range(0, N, 16384):
        q = qw[:, n0:n0 + 16384]
        b = torch.stack([(q >> (8 * i)) & 0xFF for i in range(4)], dim=1).reshape(K, -1).float() - zero
        s = sc[:, n0:n0 + 16384].float().repeat_interleave(group, dim=0)
        out[:, n0:n0 + 16384] = xf @ (b * s)
    return out


def test_int8_lm_head_sized(pkg, dev):
    """An lm_head-sized projection, K = 4096 -> N = 151,936 (1,187 column blocks of 128), with g128 scales
    and the checkpoint's zero point 128: every column against a plain PyTorch fp32 reference, and a spread of
    column blocks against the oracle."""
    K, N, M = 4096, 151936, 2
    qw, sc1 = pkg.synth.make_int8_dense(K, N, seed=9, device=dev, gen_device=dev)
    sc = (sc1.float().repeat(K // 128, 1) * torch.linspace(0.5, 1.5, K // 128, device=dev)[:, None]).to(torch.float16)
    x = pkg.synth.make_activation(M, K, seed=9, device=dev, gen_device=dev)
    y = pkg.int8_gemv(x, qw, sc)
    ref_all = _int8_torch_fp32(x, qw, sc)
    torch.cuda.synchronize()
    rel = float((y.float() - ref_all).abs().max() / ref_all.abs().max())
    assert rel < 1e-2, rel
    blocks = torch.tensor([0, 1, 500, 1000, 1186])
    cols = (blocks[:, None] * 128 + torch.arange(128)[None]).reshape(-1).to(dev)
    ref = O.int8_gemv(x.cpu(), qw[:, cols].cpu(), sc[:, cols].cpu())
    assert O.max_rel_err(y[:, cols].float().cpu(), ref) < 1e-2
