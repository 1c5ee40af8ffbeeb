"""Static per-tensor FP8 (W8A8) linears on the CPU path: quantization rules, the static-scale
checkpoint layout (scalar weight_scale / input_scale per projection, as ModelOpt writes) read
and served with FP8 projections, and the rmsnorm_quant reference modes."""
import os
import tempfile

import torch

from tests._tiny import random_prompts, tiny_llama_checkpoint
from vllm_neuron_b200.entrypoints import LLM
from vllm_neuron_b200.ops import linear as L

KW = dict(device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
          max_num_batched_tokens=64, skip_tokenizer_init=True)


def test_fp8_weight_linear_ops():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(96, 64, generator=g) * 0.05
    x = torch.randn(7, 64, generator=g)
    fw = L.FP8Weight.from_weight(w, in_scale=4.0 / 448)
    assert fw.q.dtype == torch.float8_e4m3fn and abs(fw.dequant().abs().max() - w.abs().max()) < 1e-6
    ref = x @ w.t()
    y = L.gemm_out(x, fw)
    assert ((y - ref).norm() / ref.norm()).item() < 0.06
    acc = torch.zeros(7, 96)
    L.gemm_accumulate(x, fw, acc)
    assert torch.allclose(acc, y, atol=1e-5)
    # the emulation is exactly quantize(x) @ q^T scaled
    xq = L.quantize_fp8(x, fw.in_scale)
    assert torch.allclose(y, (xq.float() @ fw.q.float().t()) * fw.in_scale * fw.w_scale, atol=1e-6)


def test_rmsnorm_quant_modes():
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(5, 64, generator=g) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(64, generator=g)).to(torch.bfloat16)
    xf = x.float()
    y = (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-5)).to(torch.bfloat16).float() * w.float()
    q, rows = L.rmsnorm_quant(x, w, 1e-5)                       # ROW
    assert rows.shape == (5,) and torch.allclose(q.float().abs().amax(-1), torch.full((5,), 448.0))
    assert ((q.float() * rows[:, None] - y).norm() / y.norm()).item() < 0.05
    q2, none = L.rmsnorm_quant(x, w, 1e-5, scale=0.01)          # STATIC
    assert none is None and ((q2.float() * 0.01 - y).norm() / y.norm()).item() < 0.05


def _static_fp8_checkpoint():
    """The tiny Llama rewritten in the static FP8 layout: e4m3 weights of every projection with
    a scalar weight_scale, and a scalar input_scale."""
    from safetensors.torch import load_file, save_file

    src, _ = tiny_llama_checkpoint()
    d = tempfile.mkdtemp(prefix="tiny_llama_fp8_")
    for f in os.listdir(src):
        if not f.endswith(".safetensors"):
            os.system(f"cp '{os.path.join(src, f)}' '{d}'")
    sd = load_file(os.path.join(src, "model.safetensors"))
    out = {}
    for k, v in sd.items():
        if k.endswith("_proj.weight"):
            s = float(v.abs().max()) / 448.0
            out[k] = (v.float() / s).clamp(-448, 448).to(torch.float8_e4m3fn)
            out[k.replace(".weight", ".weight_scale")] = torch.tensor(s, dtype=torch.float32)
            out[k.replace(".weight", ".input_scale")] = torch.tensor(6.0 / 448, dtype=torch.float32)
        else:
            out[k] = v
    save_file(out, os.path.join(d, "model.safetensors"))
    return d, src


def test_static_fp8_checkpoint_served_w8a8():
    from vllm_neuron_b200.engine.llm_engine import _static_fp8_scales

    d, src = _static_fp8_checkpoint()
    sc = _static_fp8_scales(d)
    assert sc is not None and len(sc) == 2 * 7 and abs(sc[(0, "q_proj")][1] - 6.0 / 448) < 1e-9
    prompts = random_prompts(n=3, length=20, seed=3)
    fp8 = LLM(d, **KW)
    assert fp8.engine.model.fp8_linears == 2 * 4
    assert isinstance(fp8.engine.model.layers[0].qkv, L.FP8Weight)
    ref = LLM(src, **KW).engine.prompt_logits(prompts)
    got = fp8.engine.prompt_logits(prompts)
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < 0.1, rel
    from vllm_neuron_b200.engine.sampling_params import SamplingParams

    outs = fp8.generate(prompts, SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))
    assert all(len(o.outputs[0].token_ids) > 0 for o in outs)


def test_dummy_weights_quantized_on_request():
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 256,
           "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
           "intermediate_size": 512, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
           "max_position_embeddings": 1024}
    llm = LLM(cfg, load_format="dummy", additional_config={"neuron_config": {"quantization": "fp8_static"}}, **KW)
    assert llm.engine.model.fp8_linears == 8
