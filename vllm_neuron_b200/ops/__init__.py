"""Functional ops of the framework (the B200 counterpart of ``vllm_neuron.functional``).

Every op takes preallocated outputs where it makes sense, runs the sm_100a kernel for CUDA
tensors (raising if the extension is missing) and an fp32 torch oracle for CPU tensors.
"""
from .activation import silu_mul, swiglu_oai_ref
from .attention import (AttnWork, attn_combine, build_work, dcp_local_count, paged_attention,
                        paged_attention_partial, paged_attention_ref)
from .embedding import embedding
from .linear import (gemm_accumulate, gemm_out, gemm_silu, gemm_skinny_bf16,
                     interleave_gate_up, silu_mul_ref)
from .norm import add_rmsnorm, rmsnorm, rmsnorm_ref
from .rope import cos_sin_table, rope_kv_write, rope_kv_write_ref
from . import moe
from .sampling import argmax, sample, sample_ref

__all__ = [
    "AttnWork", "add_rmsnorm", "argmax", "build_work", "cos_sin_table", "embedding",
    "gemm_accumulate", "gemm_out", "gemm_silu", "gemm_skinny_bf16", "interleave_gate_up",
    "paged_attention", "paged_attention_ref", "paged_attention_partial", "attn_combine",
    "dcp_local_count", "rmsnorm", "rmsnorm_ref", "rope_kv_write",
    "rope_kv_write_ref", "sample", "sample_ref", "silu_mul", "silu_mul_ref", "swiglu_oai_ref",
]
