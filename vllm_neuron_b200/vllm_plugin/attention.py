"""Attention backend descriptor handed to vLLM (reference: NeuronAttentionBackend,
vllm/attention/attn.py:6-35 -- a stateless spec).  The models run their own paged attention
(csrc/attn); vLLM only needs the KV-cache shape and a name."""
from __future__ import annotations


class B200AttentionBackend:
    accept_output_buffer: bool = False

    @staticmethod
    def get_name() -> str:
        return "B200_PAGED"

    @staticmethod
    def get_supported_kernel_block_sizes() -> list[int]:
        return [16, 32, 64]

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        # per layer: K and V caches of [blocks, kv_heads, block_size, head_dim]
        return (2, num_blocks, num_kv_heads, block_size, head_size)

    @staticmethod
    def get_impl_cls():
        raise NotImplementedError("the B200 models compute attention themselves")

    @staticmethod
    def get_builder_cls():
        raise NotImplementedError("the B200 worker builds its own attention metadata")
