"""Model families on the GPU (bf16, sm_100a kernels) against their fp32 CPU runs of the same
checkpoint: greedy tokens of a short generation must mostly agree."""
import tempfile

import pytest
import torch

from tests._tiny import random_prompts
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM
from vllm_neuron_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def _gpt_oss_ckpt():
    from transformers import GptOssConfig, GptOssForCausalLM

    torch.manual_seed(0)
    cfg = GptOssConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                       head_dim=64, intermediate_size=256, num_local_experts=8, num_experts_per_tok=2,
                       vocab_size=1024, sliding_window=16, max_position_embeddings=1024,
                       layer_types=["sliding_attention", "full_attention"], initializer_range=0.05)
    hf = GptOssForCausalLM(cfg).to(torch.bfloat16).eval()
    d = tempfile.mkdtemp(prefix="gptoss_gpu_")
    hf.save_pretrained(d, safe_serialization=True)
    return d


def _agree(d, tol=5e-2, **kw):
    """Prefill logits of the GPU (bf16, sm_100a kernels) against the CPU fp32 run of the same
    checkpoint, then a short greedy generation on the GPU that must not trip a device wait.
    ``tol`` is the relative logit error allowed; it is set per model from the bf16-vs-fp32
    error of the CPU reference path itself (random-init hybrids are far more sensitive)."""
    prompts = random_prompts(n=4, length=40, vocab=1024)
    cpu = LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=256, **kw)
    ref = cpu.engine.prompt_logits(prompts)
    ext().reset_status()
    gpu = LLM(d, device="cuda:0", max_num_seqs=4, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=256, **kw)
    got = gpu.engine.prompt_logits(prompts)
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < tol, rel
    assert (got.argmax(-1) == ref.argmax(-1)).float().mean() >= 0.75
    outs = gpu.generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    torch.cuda.synchronize()
    assert ext().read_status() == 0
    assert all(len(o.outputs[0].token_ids) == 8 for o in outs)


def test_gpt_oss_gpu_matches_cpu(cuda_device):
    _agree(_gpt_oss_ckpt())


def _hybrid_ckpt():
    from transformers import Qwen3_5MoeForCausalLM
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig

    torch.manual_seed(0)
    cfg = Qwen3_5MoeTextConfig(hidden_size=256, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=256, linear_key_head_dim=128, linear_value_head_dim=128,
                               linear_num_key_heads=2, linear_num_value_heads=4, linear_conv_kernel_dim=4,
                               moe_intermediate_size=128, shared_expert_intermediate_size=128, num_experts=16,
                               num_experts_per_tok=4, vocab_size=1024, max_position_embeddings=1024,
                               initializer_range=0.05, tie_word_embeddings=False,
                               rope_parameters={"rope_type": "default", "rope_theta": 10000.0,
                                                "partial_rotary_factor": 0.25})
    hf = Qwen3_5MoeForCausalLM(cfg).to(torch.bfloat16).eval()
    d = tempfile.mkdtemp(prefix="hybrid_gpu_")
    hf.save_pretrained(d, safe_serialization=True)
    return d


def test_hybrid_gpu_matches_cpu(cuda_device):
    # the CPU reference path itself differs by 0.12 between bf16 and fp32 on this checkpoint
    _agree(_hybrid_ckpt(), tol=0.25)


def test_hybrid_chunked_prefill_matches_recurrent(cuda_device):
    """The same bf16 hybrid model with its DeltaNet prefill forced to the chunked kernels and to
    the token recurrence: prefill logits of 150-token prompts (three chunks) agree."""
    from vllm_neuron_b200.models.qwen3_5 import Qwen3_5MoeForCausalLM

    d = _hybrid_ckpt()
    prompts = random_prompts(n=3, length=150, vocab=1024)
    got = {}
    for mode in ("recurrent", "chunked"):
        Qwen3_5MoeForCausalLM.deltanet_mode = mode
        try:
            llm = LLM(d, device="cuda:0", max_num_seqs=4, max_model_len=512, num_gpu_blocks=64,
                      max_num_batched_tokens=512)
            got[mode] = llm.engine.prompt_logits(prompts)
        finally:
            Qwen3_5MoeForCausalLM.deltanet_mode = "auto"
    rel = ((got["chunked"] - got["recurrent"]).norm() / got["recurrent"].norm()).item()
    assert rel < 0.1, rel
    assert ext().read_status() == 0


def test_qwen3_moe_gpu_matches_cpu(cuda_device):
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    torch.manual_seed(0)
    cfg = Qwen3MoeConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=64, intermediate_size=512, moe_intermediate_size=128, num_experts=16,
                         num_experts_per_tok=4, norm_topk_prob=True, vocab_size=1024,
                         max_position_embeddings=1024, initializer_range=0.05)
    hf = Qwen3MoeForCausalLM(cfg).to(torch.bfloat16).eval()
    d = tempfile.mkdtemp(prefix="qwen3moe_gpu_")
    hf.save_pretrained(d, safe_serialization=True)
    _agree(d)


def test_glm4_moe_gpu_matches_cpu(cuda_device):
    from transformers import Glm4MoeConfig, Glm4MoeForCausalLM

    torch.manual_seed(0)
    cfg = Glm4MoeConfig(hidden_size=256, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
                        head_dim=64, intermediate_size=512, moe_intermediate_size=128, n_routed_experts=16,
                        num_experts_per_tok=4, n_shared_experts=1, first_k_dense_replace=1,
                        routed_scaling_factor=2.5, norm_topk_prob=True, attention_bias=True,
                        use_qk_norm=True, partial_rotary_factor=0.5, vocab_size=1024,
                        max_position_embeddings=1024, initializer_range=0.05)
    hf = Glm4MoeForCausalLM(cfg).to(torch.bfloat16).eval()
    with torch.no_grad():
        for ly in hf.model.layers[1:]:
            ly.mlp.gate.e_score_correction_bias.normal_(0.0, 0.1)
    d = tempfile.mkdtemp(prefix="glm4moe_gpu_")
    hf.save_pretrained(d, safe_serialization=True)
    _agree(d)


def test_ministral3_gpu_matches_cpu(cuda_device):
    from transformers import Ministral3Config, Ministral3ForCausalLM

    torch.manual_seed(0)
    cfg = Ministral3Config(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                           head_dim=64, intermediate_size=512, vocab_size=1024, max_position_embeddings=1024,
                           initializer_range=0.05, tie_word_embeddings=False,
                           rope_parameters={"rope_type": "yarn", "rope_theta": 1000000.0, "factor": 4.0,
                                            "original_max_position_embeddings": 16, "beta_fast": 32.0,
                                            "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0,
                                            "llama_4_scaling_beta": 0.1})
    hf = Ministral3ForCausalLM(cfg).to(torch.bfloat16).eval()
    d = tempfile.mkdtemp(prefix="ministral3_gpu_")
    hf.save_pretrained(d, safe_serialization=True)
    _agree(d)


def test_qwen3_vl_gpu_matches_cpu(cuda_device):
    """Image request on the GPU (bf16 kernels, vision linears on the tcgen05 GEMM) against the
    fp32 CPU run of the same checkpoint: prompt logits close, same first tokens."""
    import numpy as np
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration

    IMG = 900
    torch.manual_seed(0)
    cfg = Qwen3VLConfig(
        text_config=dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=64, intermediate_size=512, vocab_size=1024, max_position_embeddings=1024,
                         rope_parameters={"rope_type": "default", "rope_theta": 10000.0,
                                          "mrope_section": [12, 10, 10], "mrope_interleaved": True},
                         initializer_range=0.05, tie_word_embeddings=False),
        vision_config=dict(hidden_size=64, intermediate_size=128, num_heads=2, depth=2, patch_size=8,
                           temporal_patch_size=2, spatial_merge_size=2, out_hidden_size=256,
                           num_position_embeddings=64, deepstack_visual_indexes=[0], initializer_range=0.05),
        image_token_id=IMG, vision_start_token_id=901, vision_end_token_id=902, tie_word_embeddings=False)
    hf = Qwen3VLForConditionalGeneration(cfg).to(torch.bfloat16).eval()
    d = tempfile.mkdtemp(prefix="qwen3vl_gpu_")
    hf.save_pretrained(d, safe_serialization=True)
    img = (np.random.default_rng(0).random((48, 32, 3)) * 255).astype(np.uint8)
    proc = {"min_pixels": 32 * 32, "max_pixels": 64 * 64}
    prompt = {"prompt_token_ids": [5, 6, 901, IMG, 902, 7, 8, 9], "multi_modal_data": {"image": img}}
    sp = SamplingParams(temperature=0, max_tokens=4, ignore_eos=True)
    cpu = LLM(d, device="cpu", dtype="float32", max_num_seqs=2, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=256, mm_processor_kwargs=proc, skip_tokenizer_init=True)
    ref = cpu.generate([prompt], sp)[0].outputs[0].token_ids
    ext().reset_status()
    gpu = LLM(d, device="cuda:0", max_num_seqs=2, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=256, mm_processor_kwargs=proc, skip_tokenizer_init=True)
    got = gpu.generate([prompt], sp)[0].outputs[0].token_ids
    torch.cuda.synchronize()
    assert ext().read_status() == 0
    assert got[:2] == ref[:2], (got, ref)
