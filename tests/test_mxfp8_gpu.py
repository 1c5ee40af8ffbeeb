"""MXFP8 (OCP microscaling: e4m3 values, e8m0 scale per 32 elements) on the block-scaled tensor
cores (``tcgen05.mma kind::mxf8f6f4.block_scale``) against fp32 oracles: the device quantizer
bit for bit against the host one, then every GEMM layout (decode swapped split-K fp32, prefill
bf16, transposed bf16 store, row-major fp32 split-K) against the fp32 product of the dequantized
MXFP8 operands."""
import pytest
import torch

from vllm_neuron_b200.ops import linear as L

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _x(M, K, dev, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    # rows and 32-groups of very different magnitudes exercise the per-group exponents
    x = torch.randn(M, K, generator=g) * torch.exp(torch.randn(M, K // 32, generator=g) * 2).repeat_interleave(32, 1)
    return x.to(dev, torch.bfloat16)


@pytest.mark.parametrize("M,K", [(1, 128), (7, 512), (130, 1024), (300, 4096)])
def test_quant_mx8_matches_host(cuda_device, M, K):
    from vllm_neuron_b200.ops._ext import ext

    x = _x(M, K, cuda_device, M + K)
    x[0, :32] = 0  # an all-zero group: scale 2^0
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=cuda_device)
    sf = torch.zeros(-(-M // 128), K // 128, 512, dtype=torch.uint8, device=cuda_device)
    ext().quant_mx8(x, q, sf)
    torch.cuda.synchronize()
    qr, sr = L.quantize_mx8(x.cpu())
    assert torch.equal(q.cpu().view(torch.uint8), qr.view(torch.uint8))
    assert torch.equal(sf.cpu(), L.mx8_atoms(sr))


@pytest.mark.parametrize("M,N,K", [(1, 1024, 4096), (16, 768, 1024), (33, 4096, 1024), (64, 1280, 2048),
                                   (100, 512, 512), (8, 200, 256)])
def test_mx8_decode_accumulate(cuda_device, M, N, K):
    w = L.MXFP8Weight.from_weight(_x(N, K, cuda_device, N).float() * 0.02)
    x = _x(M, K, cuda_device, M)
    ref = L._mx8_ref(x.cpu().float(), L.MXFP8Weight(w.q.cpu(), w.scales.cpu()))
    for splits in (None, 1, 4):
        acc = torch.zeros(M, N, dtype=torch.float32, device=cuda_device)
        L.gemm_accumulate(x, w, acc, splits=splits)
        torch.cuda.synchronize()
        assert _rel(acc.cpu(), ref) < 1e-4, splits


@pytest.mark.parametrize("M,N,K", [(300, 1024, 4096), (1024, 4096, 1024), (129, 384, 640), (8, 1536, 2048)])
def test_mx8_bf16_out(cuda_device, M, N, K):
    w = L.MXFP8Weight.from_weight(_x(N, K, cuda_device, N + 1).float() * 0.02)
    x = _x(M, K, cuda_device, M + 1)
    ref = L._mx8_ref(x.cpu().float(), L.MXFP8Weight(w.q.cpu(), w.scales.cpu()))
    out = L.gemm_out(x, w)
    torch.cuda.synchronize()
    assert _rel(out.cpu(), ref) < 5e-3
    # against the unquantized product: the MXFP8 rounding of both operands only
    exact = x.cpu().float() @ (_x(N, K, cuda_device, N + 1).float().cpu() * 0.02).t()
    assert _rel(out.cpu(), exact) < 0.15  # groups span e^(+-4) magnitudes: coarse e4m3 steps


def test_mx8_row_major_splitk(cuda_device):
    M, N, K = 512, 1024, 2048
    w = L.MXFP8Weight.from_weight(_x(N, K, cuda_device, 5).float() * 0.02)
    x = _x(M, K, cuda_device, 6)
    ref = L._mx8_ref(x.cpu().float(), L.MXFP8Weight(w.q.cpu(), w.scales.cpu()))
    acc = torch.zeros(M, N, dtype=torch.float32, device=cuda_device)
    L.gemm_accumulate(x, w, acc, splits=2)
    torch.cuda.synchronize()
    assert _rel(acc.cpu(), ref) < 1e-4


@pytest.mark.parametrize("T", [1, 7, 40, 300])
def test_mx8_grouped_experts(cuda_device, T):
    """MXFP8 expert stacks through the grouped block-scaled GEMM (swapped decode layout up to 64
    tokens, expert-sorted token tiles above) against the fp32 per-token oracle fed with the
    MXFP8-rounded input rows; the hidden activation's MXFP8 rounding is inside the tolerance."""
    from vllm_neuron_b200.ops import moe as MO

    E, H, I, k = 8, 512, 256, 2
    g = torch.Generator(device="cpu").manual_seed(T)
    wgu = L.MXFP8Weight.from_weight((torch.randn(E, 2 * I, H, generator=g) * 0.05).to(cuda_device))
    wd = L.MXFP8Weight.from_weight((torch.randn(E, H, I, generator=g) * 0.05).to(cuda_device))
    x = (torch.randn(T, H, generator=g)).to(cuda_device, torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(cuda_device, torch.int32)
    w = torch.rand(T, k, generator=g).to(cuda_device)
    out = MO.moe_experts(x, ids, w, wgu, wd)
    torch.cuda.synchronize()
    xq, xs = L.quantize_mx8(x.float())
    ref = MO.experts_ref(L.dequantize_mx8(xq, xs), ids, w, wgu, wd)
    assert _rel(out, ref) < 4e-2
    # against the unquantized activations too (both roundings)
    assert _rel(out, MO.experts_ref(x.float(), ids, w, wgu, wd)) < 8e-2


@pytest.mark.parametrize("T", [5, 200])
def test_mx8_padded_gptoss_experts(cuda_device, T):
    """GPT-OSS-style experts (hidden and FFN not multiples of 128, biases, clamped SwiGLU): the
    MXFP4 stacks re-encoded losslessly as MXFP8 with K and the down projection's rows zero-padded
    to 128s; the padded output rows are dropped by the combine (row stride above H)."""
    from vllm_neuron_b200.models.gpt_oss import _quant_experts
    from vllm_neuron_b200.ops import moe as MO

    E, H, I, k = 4, 320, 192, 2
    g = torch.Generator(device="cpu").manual_seed(T + 11)
    gb, gs = _quant_experts((torch.randn(E, 2 * I, H, generator=g) * 0.05).to(cuda_device))
    db, ds = _quant_experts((torch.randn(E, H, I, generator=g) * 0.05).to(cuda_device))
    w4gu, w4d = L.MXFP4Weight.from_blocks(gb, gs), L.MXFP4Weight.from_blocks(db, ds)
    wgu = L.MXFP8Weight.from_mxfp4(w4gu, k_pad=384)
    wd = L.MXFP8Weight.from_mxfp4(w4d, k_pad=256, n_pad=384)
    assert torch.equal(wgu.dequant()[..., :H], w4gu.dequant_bf16_ref().float())  # lossless
    b_gu = (torch.randn(E, 2 * I, generator=g) * 0.1).to(cuda_device, torch.bfloat16)
    b_dn = (torch.randn(E, H, generator=g) * 0.1).to(cuda_device, torch.bfloat16)
    x = torch.randn(T, H, generator=g).to(cuda_device, torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(cuda_device, torch.int32)
    w = torch.rand(T, k, generator=g).to(cuda_device)
    out = MO.moe_experts(x, ids, w, wgu, wd, b_gu=b_gu, b_down=b_dn, act=MO.ACT_GPTOSS)
    torch.cuda.synchronize()
    xq, xs = L.quantize_mx8(x.float())
    ref = MO.experts_ref(L.dequantize_mx8(xq, xs), ids, w, w4gu, w4d, b_gu, b_dn, act=MO.ACT_GPTOSS)
    assert _rel(out, ref) < 4e-2
