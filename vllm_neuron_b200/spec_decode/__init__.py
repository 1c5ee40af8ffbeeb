"""Speculative decoding: proposers (n-gram prompt lookup, EAGLE3 draft head) and the
rejection sampler that verifies their draft tokens against the target model.

Reference: vllm_neuron/vllm/spec_decode/eagle.py (EagleProposer), decorator.py (async
speculative decoding prologue/epilogue), vllm/sample/rejection_sampler.py and
nn/rejection_sampler.py (Leviathan et al., arXiv 2211.17192).
"""
from .ngram import NgramProposer
from .rejection import rejection_sample, rejection_sample_ref

__all__ = ["NgramProposer", "rejection_sample", "rejection_sample_ref"]
