"""Block-scaled FP8 weights (128 x 128 blocks, W8A16) on the tcgen05 GEMM against fp32 oracles.

The kernel streams the e4m3 weight bytes, widens each tile in shared memory with its block
scale and runs the bf16 tensor-core MMA, so its operand is exactly ``bf16(q * scale)``; the
oracle is the fp32 product of those operands.  Covers the decode regime (weights as the
128-row A operand, split-K fp32 reductions), the prefill regime (weights as B: bf16 store and
the fused SwiGLU epilogue), partial blocks (rows / K not multiples of 128) and the grouped
expert mode.
"""
import math

import pytest
import torch

from vllm_neuron_b200.ops import linear as L

pytestmark = pytest.mark.gpu


def _w(N, K, dev, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    # per-block magnitudes that differ by orders of magnitude exercise the scale indexing
    w = torch.randn(N, K, generator=g) * 0.02
    rs = torch.exp(torch.randn(-(-N // 128), 1, generator=g) * 1.5).repeat_interleave(128, 0)[:N]
    cs = torch.exp(torch.randn(1, -(-K // 128), generator=g) * 1.5).repeat_interleave(128, 1)[:, :K]
    return L.BlockFP8Weight.from_weight((w * rs * cs).to(dev))


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.fixture
def w8a16():
    prev = L.fp8_block_activations()
    L.set_fp8_block_activations("bf16")
    yield
    L.set_fp8_block_activations(prev)


@pytest.mark.parametrize("M,N,K", [(1, 1024, 4096), (16, 768, 4096), (64, 4096, 1024),
                                   (128, 3584, 8192), (64, 1280, 3584), (33, 200, 320)])
def test_block_fp8_decode_accumulate(cuda_device, w8a16, M, N, K):
    """W8A16 (exact bf16 activations, weights widened in shared memory)."""
    w = _w(N, K, cuda_device, seed=M + N)
    x = (torch.randn(M, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    acc = torch.zeros(M, N, dtype=torch.float32, device=cuda_device)
    L.gemm_accumulate(x, w, acc)
    torch.cuda.synchronize()
    ref = x.float() @ w.dequant_bf16_ref().float().t()
    assert _rel(acc, ref) < 2e-3


@pytest.mark.parametrize("M,N,K", [(1, 1024, 4096), (16, 768, 4096), (32, 4096, 1024),
                                   (7, 28672, 4096), (32, 1280, 8192), (24, 10240, 8192)])
def test_block_fp8_decode_w8a8(cuda_device, M, N, K):
    """W8A8 with per-k-block promotion: against the fp32 product of the dequantized weights and
    the dequantized per-block e4m3 activations (tight), and against the unquantized activations
    (the activation rounding only).  Repeated launches reuse the zeroed accumulator."""
    assert L.fp8_block_activations() == "fp8"
    w = _w(N, K, cuda_device, seed=M + N + 1)
    x = (torch.randn(M, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    xq, xs = L.quantize_fp8_blocks(x)
    xq_ref, xs_ref = L.quantize_fp8_blocks(x.cpu())
    assert torch.allclose(xs.cpu(), xs_ref, rtol=1e-6)
    wd = w.dequant_bf16_ref().float()
    ref_q = L.dequantize_fp8_blocks(xq, xs).float() @ wd.t()
    ref = x.float() @ wd.t()
    for _ in range(2):
        acc = torch.zeros(M, N, dtype=torch.float32, device=cuda_device)
        L.gemm_accumulate(x, w, acc)
        torch.cuda.synchronize()
        assert _rel(acc, ref_q) < 2e-3
        assert _rel(acc, ref) < 4e-2


@pytest.mark.parametrize("M,N,K", [(300, 1024, 4096), (1024, 4096, 1024), (2048, 1536, 2048),
                                   (129, 384, 640)])
def test_block_fp8_prefill_out(cuda_device, w8a16, M, N, K):
    """W8A16 prefill (weights widened in shared memory, exact bf16 activations)."""
    w = _w(N, K, cuda_device, seed=M)
    x = (torch.randn(M, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    for bn in (128, 256):
        out = L.gemm_out(x, w, bn=bn)
        torch.cuda.synchronize()
        ref = x.float() @ w.dequant_bf16_ref().float().t()
        assert _rel(out, ref) < 1e-2, bn


def test_block_fp8_prefill_silu_and_splitk(cuda_device, w8a16):
    I, K, M = 1024, 2048, 512
    g = _w(I, K, cuda_device, seed=7).dequant_bf16_ref()
    u = _w(I, K, cuda_device, seed=8).dequant_bf16_ref()
    w = L.BlockFP8Weight.from_weight(L.interleave_gate_up(g, u))
    x = (torch.randn(M, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    out = L.gemm_silu(x, w)
    torch.cuda.synchronize()
    y = x.float() @ w.dequant_bf16_ref().float().t()
    ref = L.silu_mul_ref(y, L.SILU_BLOCK)
    assert _rel(out, ref) < 1e-2
    acc = torch.zeros(M, 2 * I, dtype=torch.float32, device=cuda_device)
    L.gemm_accumulate(x, w, acc, splits=4)
    torch.cuda.synchronize()
    assert _rel(acc, y) < 2e-3


def test_block_fp8_grouped_experts(cuda_device):
    from vllm_neuron_b200.ops._ext import ext

    E, N, K, R = 4, 256, 1024, 512
    ws = [_w(N, K, cuda_device, seed=20 + e).dequant_bf16_ref() for e in range(E)]
    w = L.BlockFP8Weight.from_weight(torch.stack(ws))
    x = (torch.randn(R, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    # 128-row blocks: rows [0, 100) expert 2, [128, 300) expert 0, [384, 512) expert 3
    tiles = torch.tensor([[2, 0, 100, 0], [0, 128, 256, 0], [0, 256, 300, 0], [3, 384, 512, 0]],
                         dtype=torch.int32, device=cuda_device)
    cnt = torch.tensor([4], dtype=torch.int32, device=cuda_device)
    out = torch.zeros(R, N, dtype=torch.bfloat16, device=cuda_device)
    ext().gemm_w8(x, w.q, out, L.EPI_BF16, 128, 1, w.scales, 2, tiles, cnt)
    torch.cuda.synchronize()
    wd = w.dequant_bf16_ref().float()
    for e, a, b in ((2, 0, 100), (0, 128, 300), (3, 384, 512)):
        ref = x[a:b].float() @ wd[e].t()
        assert _rel(out[a:b], ref) < 1e-2, (e, a, b)


@pytest.mark.parametrize("M,N,K", [(300, 1024, 4096), (1024, 4096, 1024), (2048, 1536, 2048),
                                   (129, 384, 640), (4096, 28672, 8192)])
def test_block_fp8_prefill_w8a8(cuda_device, M, N, K):
    """W8A8 prefill with per-k-block promotion (tokens as the 128-row operand, 128-wide weight
    tiles, bf16 store): against the dequantized-activation oracle (tight) and the exact one."""
    assert L.fp8_block_activations() == "fp8"
    w = _w(N, K, cuda_device, seed=M + 3)
    x = (torch.randn(M, K, device=cuda_device) * 0.5).to(torch.bfloat16)
    xq, xs = L.quantize_fp8_blocks(x)
    wd = w.dequant_bf16_ref().float()
    ref_q = L.dequantize_fp8_blocks(xq, xs).float() @ wd.t()
    out = L.gemm_out(x, w)
    torch.cuda.synchronize()
    assert _rel(out, ref_q) < 5e-3
    assert _rel(out, x.float() @ wd.t()) < 4e-2
    if N % 256 == 0:  # the SwiGLU form: gate/up through the same kernel, then the activation
        y = L.gemm_silu(x, w)
        torch.cuda.synchronize()
        assert _rel(y, L.silu_mul_ref(ref_q, L.SILU_BLOCK)) < 1e-2


def test_block_fp8_linear_layer_of_model(cuda_device):
    """A Llama decoder with block-FP8 projections matches its own bf16 dequantized weights."""
    from vllm_neuron_b200.config import ModelArchConfig
    from vllm_neuron_b200.models.llama import LlamaForCausalLM

    cfg = ModelArchConfig.from_hf({"architectures": ["LlamaForCausalLM"], "hidden_size": 1024,
                                   "num_hidden_layers": 2, "num_attention_heads": 8,
                                   "num_key_value_heads": 2, "head_dim": 128,
                                   "intermediate_size": 2048, "vocab_size": 1000,
                                   "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
                                   "max_position_embeddings": 512})
    m = LlamaForCausalLM(cfg, device=cuda_device, max_tokens=512)
    m.init_random(0, std=0.05)
    n = m.quantize_block_fp8()
    assert n == 2 * 4
    for ly in m.layers:
        for name in ("qkv", "o", "gate_up", "down"):
            assert isinstance(getattr(ly, name), L.BlockFP8Weight)
    x = (torch.randn(64, 1024, device=cuda_device) * 0.5).to(torch.bfloat16)
    w = m.layers[0].gate_up
    out = L.gemm_silu(x, w)
    ref = L.silu_mul_ref(x.float() @ w.dequant_bf16_ref().float().t(), L.SILU_BLOCK)
    assert _rel(out, ref) < 1e-2
    assert math.isfinite(float(out.float().abs().max()))
