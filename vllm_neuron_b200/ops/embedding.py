"""Vocab-sharded embedding lookup (csrc/misc/norm_rope.cu ``embedding_kernel``).

Rows outside ``[vocab_start, vocab_end)`` produce zeros, so the sum over the TP group (an
all-reduce, or a reduce-scatter under sequence parallelism) yields the full embedding.
Reference: ``VocabDimShardedEmbedding`` (vllm_neuron/nn/embedding.py:23-249) and
``NF.embedding`` (functional/embedding.py:6).
"""
from __future__ import annotations

import torch

from ._ext import ext


def embedding(ids: torch.Tensor, table: torch.Tensor, vocab_start: int = 0,
              vocab_end: int | None = None, out: torch.Tensor | None = None,
              last_tok: torch.Tensor | None = None) -> torch.Tensor:
    """``ids < 0`` refer to device-resident tokens: ``id = last_tok[-id - 1]``."""
    vocab_end = table.shape[0] + vocab_start if vocab_end is None else vocab_end
    T = ids.shape[0]
    if out is None:
        out = torch.empty((T, table.shape[1]), dtype=table.dtype, device=table.device)
    if not ids.is_cuda:
        if last_tok is not None and bool((ids < 0).any()):
            ids = torch.where(ids < 0, last_tok[(-ids - 1).clamp(min=0).long()], ids)
        own = (ids >= vocab_start) & (ids < vocab_end)
        local = (ids - vocab_start).clamp(0, table.shape[0] - 1).long()
        out.copy_(table[local] * own[:, None].to(table.dtype))
        return out
    ext().embedding(ids, table, out, vocab_start, vocab_end, last_tok)
    return out
