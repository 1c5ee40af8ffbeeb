"""Shared helpers for CPU tests: the tiny Llama-3 configuration of the plumbing benchmark
(2 layers, hidden 256, 4 query / 2 KV heads, head_dim 64, FFN 512, vocab 32000) saved as an
HF checkpoint with N(0, 0.02) weights from seed 0."""
import functools
import tempfile

import torch


def tiny_llama_config(**over):
    from transformers import LlamaConfig

    kw = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
              head_dim=64, intermediate_size=512, rms_norm_eps=1e-5, rope_theta=500000.0,
              vocab_size=32000, tie_word_embeddings=False, max_position_embeddings=2048,
              initializer_range=0.02)
    kw.update(over)
    return LlamaConfig(**kw)


@functools.lru_cache(maxsize=4)
def tiny_llama_checkpoint(seed: int = 0, num_key_value_heads: int = 2):
    from transformers import LlamaForCausalLM

    torch.manual_seed(seed)
    hf = LlamaForCausalLM(tiny_llama_config(num_key_value_heads=num_key_value_heads)).float().eval()
    d = tempfile.mkdtemp(prefix="tiny_llama_")
    hf.save_pretrained(d, safe_serialization=True)
    return d, hf


def random_prompts(n=4, length=32, vocab=32000, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (length,), generator=g).tolist() for _ in range(n)]
