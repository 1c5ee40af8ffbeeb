"""MXFP4 experts (e2m1 + e8m0 per 32) on the tcgen05 grouped GEMM (W4A16) against fp32 oracles.

The packed bytes are widened in shared memory with each block's power-of-two scale, which is
exact in bf16, so the oracle is the fp32 product with the dequantized weights.  Covers the
GPT-OSS expert shapes (gate/up rows 2 I, down rows H not a multiple of 128), a decode-sized
and a prefill-sized tile list, and a GPT-OSS MoE block whose experts are MXFP4Weight stacks.
"""
import pytest
import torch

from vllm_neuron_b200.ops import linear as L
from vllm_neuron_b200.ops import moe as M
from vllm_neuron_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def _mx(E, N, K, dev, seed):
    from vllm_neuron_b200.models.gpt_oss import quant_mxfp4

    g = torch.Generator().manual_seed(seed)
    w = torch.randn(E, N, K, generator=g) * 0.05
    b, s = zip(*(quant_mxfp4(w[e]) for e in range(E)))
    return L.MXFP4Weight.from_blocks(torch.stack(b).to(dev), torch.stack(s).to(dev))


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize("N,K,rows", [(5760, 2880, 40), (2880, 2880, 600), (1024, 512, 300)])
def test_mxfp4_grouped_gemm(cuda_device, N, K, rows):
    E = 4
    w = _mx(E, N, K, cuda_device, seed=N + rows)
    x = (torch.randn(rows, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    # tile list: expert e takes rows [first, end) of 128-row blocks
    bounds = torch.linspace(0, rows, E + 1).long().tolist()
    tiles = []
    for e in range(E):
        a, b = bounds[e], bounds[e + 1]
        for r in range(a, b, 128):  # a tile multiplies rows [r, r + 128), stores rows below end
            tiles.append([e, r, min(b, r + 128), 0])
    gt = torch.tensor(tiles, dtype=torch.int32, device=cuda_device)
    cnt = torch.tensor([len(tiles)], dtype=torch.int32, device=cuda_device)
    out = torch.zeros(rows, N, dtype=torch.bfloat16, device=cuda_device)
    for bn in (128, 256):
        out.zero_()
        ext().gemm_w8(x, w.q, out, L.EPI_BF16, bn, 1, w.scales, 4, gt, cnt)
        torch.cuda.synchronize()
        wd = w.dequant().float()
        for e in range(E):
            a, b = bounds[e], bounds[e + 1]
            if b > a:
                ref = x[a:b].float() @ wd[e].t()
                assert _rel(out[a:b], ref) < 1e-2, (e, bn)


@pytest.mark.parametrize("T", [8, 64, 300])
def test_mxfp4_moe_block_gptoss(cuda_device, T):
    E, H, I, k = 8, 2880, 2880, 4
    w_gu = _mx(E, 2 * I, H, cuda_device, seed=1)
    w_dn = _mx(E, H, I, cuda_device, seed=2)
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16).to(cuda_device)
    router = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    rb = torch.zeros(E, device=cuda_device)
    b_gu = (torch.randn(E, 2 * I, generator=g) * 0.1).to(torch.bfloat16).to(cuda_device)
    b_dn = (torch.randn(E, H, generator=g) * 0.1).to(torch.bfloat16).to(cuda_device)
    out = M.moe_block(x, router, w_gu, w_dn, k, M.ROUTE_TOPK_SOFTMAX, router_b=rb, b_gu=b_gu, b_down=b_dn,
                      act=M.ACT_GPTOSS, alpha=1.702, limit=7.0)
    torch.cuda.synchronize()
    ref = M.moe_block(x.cpu(), router.cpu(), L.MXFP4Weight(w_gu.q.cpu(), w_gu.scales.cpu()),
                      L.MXFP4Weight(w_dn.q.cpu(), w_dn.scales.cpu()), k, M.ROUTE_TOPK_SOFTMAX,
                      router_b=rb.cpu(), b_gu=b_gu.cpu(), b_down=b_dn.cpu(), act=M.ACT_GPTOSS,
                      alpha=1.702, limit=7.0)
    assert _rel(out.cpu(), ref) < 3e-2


@pytest.mark.parametrize("N,K,bn", [(5760, 2880, 16), (2880, 2880, 64), (1024, 512, 32)])
def test_mxfp4_grouped_swapped(cuda_device, N, K, bn):
    """Decode-size experts: weights as the 128-row operand, each expert's <= bn tokens as the N
    tile, transposed store (the swapped grouped mode of the tcgen05 GEMM)."""
    E = 6
    w = _mx(E, N, K, cuda_device, seed=N + bn)
    counts = [min(bn, c) for c in (1, 0, bn, 3, bn - 1, 2)]  # expert 1 has no tokens
    rows = sum(counts)
    x = (torch.randn(rows, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    tiles, r = [], 0
    for e, c in enumerate(counts):
        if c:
            tiles.append([e, r, r + c, 0])
        r += c
    gt = torch.tensor(tiles + [[0, 0, 0, 0]] * 3, dtype=torch.int32, device=cuda_device)  # spare entries
    cnt = torch.tensor([len(tiles)], dtype=torch.int32, device=cuda_device)
    out = torch.full((rows, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    ext().gemm_w8(w.q, x, out, L.EPI_BF16_T, bn, 1, w.scales, 3, gt, cnt)
    torch.cuda.synchronize()
    wd = w.dequant().float()
    r = 0
    for e, c in enumerate(counts):
        if c:
            ref = x[r:r + c].float() @ wd[e].t()
            assert _rel(out[r:r + c], ref) < 1e-2, e
        r += c
    assert not torch.isnan(out).any()
