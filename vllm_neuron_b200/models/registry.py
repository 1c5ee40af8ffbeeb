"""Architecture name -> model class (reference: vllm_neuron/model/registry.py:11-38)."""
from __future__ import annotations

import importlib

_MODELS = {
    "LlamaForCausalLM": ("vllm_neuron_b200.models.llama", "LlamaForCausalLM"),
    "MistralForCausalLM": ("vllm_neuron_b200.models.llama", "LlamaForCausalLM"),
    "MinistralForCausalLM": ("vllm_neuron_b200.models.llama", "LlamaForCausalLM"),
    "Ministral3ForCausalLM": ("vllm_neuron_b200.models.llama", "LlamaForCausalLM"),
    "Qwen3ForCausalLM": ("vllm_neuron_b200.models.llama", "LlamaForCausalLM"),
    "Qwen2ForCausalLM": ("vllm_neuron_b200.models.llama", "LlamaForCausalLM"),
    # embedding backbones (pooling through LLM.embed)
    "Qwen3Model": ("vllm_neuron_b200.models.llama", "LlamaForCausalLM"),
    "LlamaModel": ("vllm_neuron_b200.models.llama", "LlamaForCausalLM"),
    "GptOssForCausalLM": ("vllm_neuron_b200.models.gpt_oss", "GptOssForCausalLM"),
    "Qwen3MoeForCausalLM": ("vllm_neuron_b200.models.qwen_moe", "Qwen3MoeForCausalLM"),
    "Qwen2MoeForCausalLM": ("vllm_neuron_b200.models.qwen_moe", "Qwen2MoeForCausalLM"),
    "Qwen3VLForConditionalGeneration": ("vllm_neuron_b200.models.qwen3_vl", "Qwen3VLForConditionalGeneration"),
    "Glm4MoeForCausalLM": ("vllm_neuron_b200.models.glm4_moe", "Glm4MoeForCausalLM"),
    "SyntheticForCausalLM": ("vllm_neuron_b200.models.synthetic", "SyntheticForCausalLM"),
    "Qwen3_5MoeForCausalLM": ("vllm_neuron_b200.models.qwen3_5", "Qwen3_5MoeForCausalLM"),
    "Qwen3_5MoeForConditionalGeneration": ("vllm_neuron_b200.models.qwen3_5", "Qwen3_5MoeForCausalLM"),
}


def register_model(arch: str, module: str, cls: str):
    _MODELS[arch] = (module, cls)


def get_models() -> dict[str, tuple[str, str]]:
    return dict(_MODELS)


def resolve(arch_names) -> type:
    for a in arch_names:
        if a in _MODELS:
            mod, cls = _MODELS[a]
            return getattr(importlib.import_module(mod), cls)
    raise ValueError(f"unsupported architectures {list(arch_names)}; supported: {sorted(_MODELS)}")
