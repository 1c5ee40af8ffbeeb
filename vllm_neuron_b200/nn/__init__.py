"""Tensor-parallel layers over the framework's kernels, for building models outside the
bundled families (reference: vllm_neuron/nn: ``ColumnParallelLinear`` cpl.py:27-143,
``RowParallelLinear`` rpl.py:23-154, ``VocabDimShardedEmbedding`` / ``EmbedDimShardedEmbedding``
embedding.py:23-433, ``Sampler`` sampler.py:13-169, ``rejection_sampler`` rejection_sampler.py:12).

Every layer takes a :class:`~vllm_neuron_b200.parallel.comm.GroupComm` (the TP group); with
``comm.world == 1`` it is a plain layer.  Weights are stored as this rank's shard in bf16 and
multiplied by the tcgen05 GEMM (`csrc/gemm`) on a B200, by torch matmul on the CPU.
"""
from .layers import (ColumnParallelLinear, EmbedDimShardedEmbedding, MergedColumnParallelLinear,
                     QKVParallelLinear, RowParallelLinear, VocabParallelEmbedding, shard_range)
from .sampler import Sampler, rejection_sampler

__all__ = ["ColumnParallelLinear", "MergedColumnParallelLinear", "QKVParallelLinear",
           "RowParallelLinear", "VocabParallelEmbedding", "EmbedDimShardedEmbedding", "Sampler",
           "rejection_sampler", "shard_range"]
