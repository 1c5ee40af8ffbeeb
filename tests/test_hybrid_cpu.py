"""Hybrid gated-DeltaNet + gated-attention MoE (Qwen3.5/3.6 family, text) on CPU in fp32 against
HF transformers, including chunked prefill (the recurrent and conv states carry across
chunks) and the op-level oracles of the DeltaNet kernels."""
import tempfile

import torch

from tests._tiny import random_prompts
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM
from vllm_neuron_b200.ops import deltanet as DN


def _tiny_hybrid(seed=0):
    from transformers import Qwen3_5MoeForCausalLM
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig

    torch.manual_seed(seed)
    cfg = Qwen3_5MoeTextConfig(hidden_size=128, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=64, linear_key_head_dim=128, linear_value_head_dim=128,
                               linear_num_key_heads=1, linear_num_value_heads=2, linear_conv_kernel_dim=4,
                               moe_intermediate_size=32, shared_expert_intermediate_size=32, num_experts=8,
                               num_experts_per_tok=2, vocab_size=512, max_position_embeddings=512,
                               initializer_range=0.05, tie_word_embeddings=False,
                               rope_parameters={"rope_type": "default", "rope_theta": 10000.0,
                                                "partial_rotary_factor": 0.25})
    hf = Qwen3_5MoeForCausalLM(cfg).float().eval()
    with torch.no_grad():
        for n, prm in hf.named_parameters():
            if "norm" in n and "linear_attn.norm" not in n:
                prm.normal_(0.0, 0.1)  # exercise the (1 + w) norm convention
    d = tempfile.mkdtemp(prefix="tiny_hybrid_")
    hf.save_pretrained(d, safe_serialization=True)
    return d, hf


def _hf_greedy(hf, prompt, n):
    ids = torch.tensor([prompt])
    out = []
    with torch.no_grad():
        for _ in range(n):
            nxt = int(hf(ids).logits[0, -1].argmax())
            out.append(nxt)
            ids = torch.cat([ids, torch.tensor([[nxt]])], 1)
    return out


def test_hybrid_generate_matches_hf():
    d, hf = _tiny_hybrid()
    prompts = random_prompts(n=3, length=30, vocab=512)
    ref = [_hf_greedy(hf, p, 8) for p in prompts]
    for chunk in (256, 16):  # whole-prompt prefill, then chunked prefill across steps
        llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
                  max_num_batched_tokens=chunk)
        outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
        assert [o.outputs[0].token_ids for o in outs] == ref, chunk


def test_conv1d_ref_matches_full_sequence():
    C, K = 6, 4
    x = torch.randn(10, C)
    w = torch.randn(C, K)
    full = torch.nn.functional.silu(torch.nn.functional.conv1d(x.t()[None], w[:, None, :], padding=K - 1,
                                                               groups=C)[0, :, :10].t())
    state = torch.zeros(2, C, K - 1)
    slots = torch.tensor([1], dtype=torch.int32)
    a = DN.causal_conv1d_ref(x[:7], w, torch.tensor([0, 7]), torch.tensor([7]), slots, state)
    b = DN.causal_conv1d_ref(x[7:], w, torch.tensor([0, 3]), torch.tensor([10]), slots, state)
    assert torch.allclose(torch.cat([a, b]), full, atol=1e-5)
