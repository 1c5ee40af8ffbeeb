"""Static FP8 (W8A8) GEMM and activation quantization kernels on the GPU against the exact torch
emulation (the same quantized operands multiplied in fp32), plus a model served W8A8."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_neuron_b200.ops import linear as L
from vllm_neuron_b200.ops._ext import ext


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


def _case(dev, M, N, K):
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) * 0.05).to(torch.bfloat16)
    fw = L.FP8Weight.from_weight(w, in_scale=float(x.float().abs().max()) / 448)
    xq = L.quantize_fp8(x, fw.in_scale)
    ref = (xq.float() @ fw.q.float().t()) * fw.in_scale * fw.w_scale
    return x, fw, ref


@pytest.mark.parametrize("M,N,K", [(300, 384, 256), (1000, 4096, 4096), (129, 6144, 4096), (64, 1000, 144)])
def test_fp8_gemm_wide(cuda_device, M, N, K):
    x, fw, ref = _case(cuda_device, M, N, K)
    for bn in (128, 256):
        assert _rel_err(L.gemm_out(x, fw, bn=bn), ref) < 1e-2
    acc = torch.zeros(M, N, device=cuda_device)
    L.gemm_accumulate(x, fw, acc) if M <= L.SKINNY_MAX else L.gemm_accumulate(x, fw, acc, splits=3)
    assert _rel_err(acc, ref) < 1e-3


@pytest.mark.parametrize("M", [1, 7, 64, 128])
@pytest.mark.parametrize("N,K", [(6144, 4096), (4096, 14336)])
def test_fp8_gemm_skinny_splitk(cuda_device, M, N, K):
    x, fw, ref = _case(cuda_device, M, N, K)
    acc = torch.zeros(M, N, device=cuda_device)
    L.gemm_accumulate(x, fw, acc)
    assert _rel_err(acc, ref) < 1e-3
    acc.zero_()
    L.gemm_accumulate(x, fw, acc, splits=3)
    assert _rel_err(acc, ref) < 1e-3


def test_fp8_gemm_silu(cuda_device):
    M, I, K = 300, 1024, 2048
    x = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    g = (torch.randn(I, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    u = (torch.randn(I, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    fw = L.FP8Weight.from_weight(L.interleave_gate_up(g, u), in_scale=float(x.float().abs().max()) / 448)
    xq = L.quantize_fp8(x, fw.in_scale)
    y = (xq.float() @ fw.q.float().t()) * fw.in_scale * fw.w_scale
    ref = L.silu_mul_ref(y, L.SILU_BLOCK)
    assert _rel_err(L.gemm_silu(x, fw), ref) < 1e-2


def test_quant_kernels_match_torch(cuda_device):
    x = (torch.randn(37, 4096, device=cuda_device) * 5).to(torch.bfloat16)
    got = L.quantize_fp8(x, 0.02)
    want = (x.float().cpu() * torch.tensor(1 / 0.02)).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert (got.cpu().view(torch.uint8) == want.view(torch.uint8)).float().mean() > 0.999
    w = (1 + 0.1 * torch.randn(4096, device=cuda_device)).to(torch.bfloat16)
    for scale in (None, 0.01):
        q, rows = L.rmsnorm_quant(x, w, 1e-5, scale)
        qr, rr = L.rmsnorm_quant(x.cpu(), w.cpu(), 1e-5, scale)
        deq = q.float().cpu() * (rows.cpu()[:, None] if rows is not None else scale)
        deq_r = qr.float() * (rr[:, None] if rr is not None else scale)
        assert _rel_err(deq, deq_r) < 1e-2


def test_w8a8_model_serves(cuda_device):
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 512,
           "num_hidden_layers": 2, "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 64,
           "intermediate_size": 1024, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
           "max_position_embeddings": 2048}
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (37, 150, 90)]
    res = {}
    for q in (None, "fp8_static"):
        llm = LLM(cfg, max_num_seqs=4, max_model_len=512, num_gpu_blocks=128, load_format="dummy",
                  device="cuda:0", skip_tokenizer_init=True,
                  additional_config={"neuron_config": {"quantization": q}} if q else None)
        res[q] = llm.engine.prompt_logits(prompts)
        outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
        assert all(len(o.outputs[0].token_ids) == 8 for o in outs)
        if q:
            assert llm.engine.model.fp8_linears == 8
        llm.shutdown()
    assert _rel_err(res["fp8_static"], res[None]) < 0.2
