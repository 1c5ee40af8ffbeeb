"""MoE kernels on the GPU against fp32 torch oracles: router top-k (three orderings), the
grouped tcgen05 GEMM through the whole routed-experts block (SiLU and GPT-OSS activations,
biases, expert-parallel shards)."""
import pytest
import torch

from vllm_neuron_b200.ops import moe as M
from vllm_neuron_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _status(cuda_device):
    torch.manual_seed(0)
    ext().reset_status()
    yield
    torch.cuda.synchronize()
    assert ext().read_status() == 0


@pytest.mark.parametrize("mode,renorm", [(M.ROUTE_TOPK_SOFTMAX, True), (M.ROUTE_SOFTMAX_TOPK, True),
                                         (M.ROUTE_SOFTMAX_TOPK, False), (M.ROUTE_SIGMOID_TOPK, True),
                                         (M.ROUTE_SIGMOID_BIAS_TOPK, True), (M.ROUTE_SIGMOID_BIAS_TOPK, False)])
@pytest.mark.parametrize("E,k", [(32, 4), (256, 8), (128, 1)])
def test_route(cuda_device, mode, renorm, E, k):
    T = 300
    logits = (torch.randn(T, E, device=cuda_device) * 2).to(torch.bfloat16)
    bias = torch.randn(E, device=cuda_device) * 0.1
    scale = 2.5 if mode == M.ROUTE_SIGMOID_BIAS_TOPK else 1.0
    ids, w = M.route(logits, k, mode, renorm, bias, scale=scale)
    rid, rw = M.route_ref(logits, k, mode, renorm, bias, scale)
    # compare as sets per token (the order of equal scores may differ)
    s_ids, o = torch.sort(ids.long(), -1)
    s_rid, ro = torch.sort(rid.long(), -1)
    assert (s_ids == s_rid).float().mean() > 0.99
    same = (s_ids == s_rid).all(-1)
    assert torch.allclose(torch.gather(w, 1, o)[same], torch.gather(rw, 1, ro)[same], atol=2e-3 * scale)


@pytest.mark.parametrize("T", [1, 7, 64, 300])
@pytest.mark.parametrize("kind", ["qwen", "gptoss", "gptoss_ep"])
def test_moe_block(cuda_device, T, kind):
    if kind == "qwen":
        E, k, H, I, mode, act, biases, e_start, e_local = 64, 8, 512, 256, M.ROUTE_SOFTMAX_TOPK, M.ACT_SILU, False, 0, 64
    else:
        E, k, H, I, mode, act, biases = 32, 4, 2880 // 4, 2880 // 4, M.ROUTE_TOPK_SOFTMAX, M.ACT_GPTOSS, True
        e_start, e_local = (8, 16) if kind == "gptoss_ep" else (0, 32)
    g = torch.Generator(device=cuda_device).manual_seed(1)
    x = torch.randn(T, H, device=cuda_device, generator=g).to(torch.bfloat16)
    rw = (torch.randn(E, H, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    rb = torch.randn(E, device=cuda_device, generator=g) * 0.1 if biases else None
    w_gu = (torch.randn(e_local, 2 * I, H, device=cuda_device, generator=g) * H ** -0.5).to(torch.bfloat16)
    w_dn = (torch.randn(e_local, H, I, device=cuda_device, generator=g) * I ** -0.5).to(torch.bfloat16)
    b_gu = (torch.randn(e_local, 2 * I, device=cuda_device, generator=g) * 0.1).to(torch.bfloat16) if biases else None
    b_dn = (torch.randn(e_local, H, device=cuda_device, generator=g) * 0.1).to(torch.bfloat16) if biases else None
    ws = M.MoEWorkspace.create(512, k, E, e_local, H, I, cuda_device)
    out = M.moe_block(x, rw, w_gu, w_dn, k, mode, True, rb, b_gu, b_dn, act, e_start=e_start, ws=ws)
    logits = ws.logits[:T, :E]
    ids, w = M.route_ref(logits, k, mode, True, rb)
    ref = M.experts_ref(x, ids, w, w_gu, w_dn, b_gu, b_dn, act, e_start=e_start)
    assert _rel_err(out, ref) < 2e-2
    # a second call with other tokens reuses the workspace
    x2 = torch.randn(T, H, device=cuda_device, generator=g).to(torch.bfloat16)
    out2 = M.moe_block(x2, rw, w_gu, w_dn, k, mode, True, rb, b_gu, b_dn, act, e_start=e_start, ws=ws)
    ids2, w2 = M.route_ref(ws.logits[:T, :E], k, mode, True, rb)
    ref2 = M.experts_ref(x2, ids2, w2, w_gu, w_dn, b_gu, b_dn, act, e_start=e_start)
    assert _rel_err(out2, ref2) < 2e-2


@pytest.mark.parametrize("T", [3, 200])
def test_moe_block_shared_expert(cuda_device, T):
    E, k, H, I = 64, 8, 512, 256
    g = torch.Generator(device=cuda_device).manual_seed(2)
    x = torch.randn(T, H, device=cuda_device, generator=g).to(torch.bfloat16)
    rw = (torch.randn(E + 1, H, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    w_gu = (torch.randn(E, 2 * I, H, device=cuda_device, generator=g) * H ** -0.5).to(torch.bfloat16)
    w_dn = (torch.randn(E, H, I, device=cuda_device, generator=g) * I ** -0.5).to(torch.bfloat16)
    s_gu = (torch.randn(2 * I, H, device=cuda_device, generator=g) * H ** -0.5).to(torch.bfloat16)
    s_dn = (torch.randn(H, I, device=cuda_device, generator=g) * I ** -0.5).to(torch.bfloat16)
    ws = M.MoEWorkspace.create(256, k, E, E, H, I, cuda_device, shared_inter=I)
    out = M.moe_block(x, rw, w_gu, w_dn, k, M.ROUTE_SOFTMAX_TOPK, True, ws=ws, num_experts=E,
                      shared_gu=s_gu, shared_down=s_dn)
    logits = ws.logits[:T, :E + 1]
    ids, w = M.route_ref(logits[:, :E], k, M.ROUTE_SOFTMAX_TOPK, True)
    ref = M.experts_ref(x, ids, w, w_gu, w_dn) + torch.sigmoid(logits[:, E:].float()) * M.shared_expert_ref(x, s_gu, s_dn)
    assert _rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("T", [1, 5, 32])
def test_moe_block_mxfp4_decode(cuda_device, T):
    """GPT-OSS-style block with MXFP4 experts: the fp4 decode kernel against the fp32 oracle of
    the same (dequantized) weights."""
    from vllm_neuron_b200.models.gpt_oss import dequant_mxfp4, quant_mxfp4

    E, k, H, I = 32, 4, 1536, 1344  # K of both matmuls a multiple of 64
    g = torch.Generator(device=cuda_device).manual_seed(3)
    x = torch.randn(T, H, device=cuda_device, generator=g).to(torch.bfloat16)
    rw = (torch.randn(E, H, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    gu_b, gu_s = quant_mxfp4(torch.randn(E, 2 * I, H, generator=torch.Generator().manual_seed(4)) * H ** -0.5)
    dn_b, dn_s = quant_mxfp4(torch.randn(E, H, I, generator=torch.Generator().manual_seed(5)) * I ** -0.5)
    w_gu = dequant_mxfp4(gu_b, gu_s).to(cuda_device)
    w_dn = dequant_mxfp4(dn_b, dn_s).to(cuda_device)
    fp4_gu = M.pack_mxfp4(gu_b, gu_s).to(cuda_device)
    fp4_dn = M.pack_mxfp4(dn_b, dn_s).to(cuda_device)
    ws = M.MoEWorkspace.create(64, k, E, E, H, I, cuda_device)
    out = M.moe_block(x, rw, w_gu, w_dn, k, M.ROUTE_TOPK_SOFTMAX, act=M.ACT_GPTOSS, ws=ws,
                      fp4_gu=fp4_gu, fp4_down=fp4_dn)
    ids, w = M.route_ref(ws.logits[:T, :E], k, M.ROUTE_TOPK_SOFTMAX)
    ref = M.experts_ref(x, ids, w, w_gu, w_dn, act=M.ACT_GPTOSS)
    assert _rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("T", [3, 200])
def test_moe_block_glm_routing_ungated_shared(cuda_device, T):
    """GLM-4.5 MoE block: biased-sigmoid routing, routed scaling factor, ungated shared expert."""
    E, k, H, I = 64, 8, 512, 256
    g = torch.Generator(device=cuda_device).manual_seed(5)
    x = torch.randn(T, H, device=cuda_device, generator=g).to(torch.bfloat16)
    rw = (torch.randn(E, H, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    rb = torch.randn(E, device=cuda_device, generator=g) * 0.1
    w_gu = (torch.randn(E, 2 * I, H, device=cuda_device, generator=g) * H ** -0.5).to(torch.bfloat16)
    w_dn = (torch.randn(E, H, I, device=cuda_device, generator=g) * I ** -0.5).to(torch.bfloat16)
    s_gu = (torch.randn(2 * I, H, device=cuda_device, generator=g) * H ** -0.5).to(torch.bfloat16)
    s_dn = (torch.randn(H, I, device=cuda_device, generator=g) * I ** -0.5).to(torch.bfloat16)
    ws = M.MoEWorkspace.create(256, k, E, E, H, I, cuda_device, shared_inter=I)
    out = M.moe_block(x, rw, w_gu, w_dn, k, M.ROUTE_SIGMOID_BIAS_TOPK, True, rb, ws=ws, num_experts=E,
                      shared_gu=s_gu, shared_down=s_dn, routed_scale=2.5, shared_gated=False)
    ids, w = M.route_ref(ws.logits[:T, :E], k, M.ROUTE_SIGMOID_BIAS_TOPK, True, rb, 2.5)
    ref = M.experts_ref(x, ids, w, w_gu, w_dn) + M.shared_expert_ref(x, s_gu, s_dn)
    assert _rel_err(out, ref) < 2e-2
