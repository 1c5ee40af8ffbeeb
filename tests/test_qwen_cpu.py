"""Qwen families on CPU (fp32) against HF transformers: Qwen3 (QK-norm dense), Qwen3-MoE
(softmax top-k, renormalised) and Qwen2-MoE (shared expert with sigmoid gate)."""
import tempfile

import pytest
import torch

from tests._tiny import random_prompts
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM


def _hf_greedy(hf, prompt, n):
    ids = torch.tensor([prompt])
    out = []
    with torch.no_grad():
        for _ in range(n):
            nxt = int(hf(ids).logits[0, -1].argmax())
            out.append(nxt)
            ids = torch.cat([ids, torch.tensor([[nxt]])], 1)
    return out


def _save(hf):
    d = tempfile.mkdtemp(prefix="tiny_qwen_")
    hf.save_pretrained(d, safe_serialization=True)
    return d


def _check(d, hf, vocab):
    prompts = random_prompts(n=3, length=24, vocab=vocab)
    llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=64)
    outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert o.outputs[0].token_ids == _hf_greedy(hf, p, 8)


def test_qwen3_dense():
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen3Config(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=16, intermediate_size=128, vocab_size=512, max_position_embeddings=256,
                      initializer_range=0.05, tie_word_embeddings=False)
    hf = Qwen3ForCausalLM(cfg).float().eval()
    _check(_save(hf), hf, 512)


@pytest.mark.parametrize("renorm", [True, False])
def test_qwen3_moe(renorm):
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    torch.manual_seed(1)
    cfg = Qwen3MoeConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=16, intermediate_size=128, moe_intermediate_size=32, num_experts=8,
                         num_experts_per_tok=2, norm_topk_prob=renorm, vocab_size=512,
                         max_position_embeddings=256, initializer_range=0.05)
    hf = Qwen3MoeForCausalLM(cfg).float().eval()
    _check(_save(hf), hf, 512)


def test_qwen2_moe_shared_expert():
    from transformers import Qwen2MoeConfig, Qwen2MoeForCausalLM

    torch.manual_seed(2)
    cfg = Qwen2MoeConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                         intermediate_size=128, moe_intermediate_size=32, shared_expert_intermediate_size=48,
                         num_experts=8, num_experts_per_tok=2, norm_topk_prob=False, vocab_size=512,
                         max_position_embeddings=256, initializer_range=0.05, qkv_bias=True)
    hf = Qwen2MoeForCausalLM(cfg).float().eval()
    _check(_save(hf), hf, 512)


def test_qwen3_embedding_pooling():
    """Qwen3-Embedding style: encoder-only Qwen3Model checkpoint, LAST-token pooling, L2 norm."""
    from transformers import Qwen3Config, Qwen3Model

    torch.manual_seed(3)
    cfg = Qwen3Config(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=16, intermediate_size=128, vocab_size=512, max_position_embeddings=256,
                      initializer_range=0.05)
    hf = Qwen3Model(cfg).float().eval()
    d = _save(hf)
    prompts = random_prompts(n=3, length=17, vocab=512)
    llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=128)
    got = torch.tensor([o.embedding for o in llm.embed(prompts)])
    with torch.no_grad():
        ref = torch.stack([hf(torch.tensor([p])).last_hidden_state[0, -1] for p in prompts])
    ref = torch.nn.functional.normalize(ref, dim=-1)
    assert torch.allclose(got, ref, atol=2e-3)  # the QK-norm output is rounded to bf16 as on the GPU


def test_ministral3_yarn_and_query_temperature():
    """Ministral-3 text model: YaRN (mscale / mscale_all_dim) and the position-dependent query
    scale 1 + beta * log(1 + floor(pos / original_max)); a small original_max makes the scale
    change inside the prompts."""
    from transformers import Ministral3Config, Ministral3ForCausalLM

    torch.manual_seed(4)
    cfg = Ministral3Config(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                           head_dim=16, intermediate_size=128, vocab_size=512, max_position_embeddings=256,
                           initializer_range=0.05, tie_word_embeddings=False,
                           rope_parameters={"rope_type": "yarn", "rope_theta": 1000000.0, "factor": 4.0,
                                            "original_max_position_embeddings": 8, "beta_fast": 32.0,
                                            "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0,
                                            "llama_4_scaling_beta": 0.5})
    hf = Ministral3ForCausalLM(cfg).float().eval()
    _check(_save(hf), hf, 512)


def test_glm4_moe():
    """GLM-4.5-style MoE: dense first layer, biased-sigmoid routing with routed scaling,
    ungated shared expert, q/k/v bias, partial rotary, QK-norm."""
    from transformers import Glm4MoeConfig, Glm4MoeForCausalLM

    torch.manual_seed(6)
    cfg = Glm4MoeConfig(hidden_size=64, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
                        head_dim=16, intermediate_size=128, moe_intermediate_size=32, n_routed_experts=8,
                        num_experts_per_tok=2, n_shared_experts=1, first_k_dense_replace=1,
                        routed_scaling_factor=2.5, norm_topk_prob=True, n_group=1, topk_group=1,
                        attention_bias=True, use_qk_norm=True, partial_rotary_factor=0.5,
                        vocab_size=512, max_position_embeddings=256, initializer_range=0.05,
                        tie_word_embeddings=False)
    hf = Glm4MoeForCausalLM(cfg).float().eval()
    with torch.no_grad():  # non-zero correction bias and attention biases
        for ly in hf.model.layers[1:]:
            ly.mlp.gate.e_score_correction_bias.normal_(0.0, 0.1)
        for ly in hf.model.layers:
            for m in (ly.self_attn.q_proj, ly.self_attn.k_proj, ly.self_attn.v_proj):
                m.bias.normal_(0.0, 0.05)
    _check(_save(hf), hf, 512)
