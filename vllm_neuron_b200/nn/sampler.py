"""Sampling layers (reference: Sampler, nn/sampler.py:13-169; rejection_sampler,
nn/rejection_sampler.py:12)."""
from __future__ import annotations

import torch

from .. import ops
from ..ops import sampling as S
from ..parallel.comm import SINGLE, GroupComm


class Sampler(torch.nn.Module):
    """Per-row temperature / top-k / top-p / min-p sampling on the device (csrc sampling
    kernel), after an optional structured-output bitmask.  Vocabulary-sharded logits are
    all-gathered over ``comm`` first (the LM head of a TP model is vocab-parallel).

    ``forward(logits [B, V_local], temperature [B], top_k [B], top_p [B], seeds [B],
    offsets [B], min_p=None, bitmask=None)`` -> token ids ``[B]`` int32 (greedy where
    temperature <= 0)."""

    def __init__(self, comm: GroupComm = SINGLE, vocab_size: int | None = None):
        super().__init__()
        self.comm = comm
        self.vocab_size = vocab_size

    def forward(self, logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                top_p: torch.Tensor, seeds: torch.Tensor, offsets: torch.Tensor,
                min_p: torch.Tensor | None = None, bitmask: torch.Tensor | None = None,
                out_logprob: torch.Tensor | None = None) -> torch.Tensor:
        if self.comm.world > 1:
            logits = self.comm.all_gather(logits.contiguous(), dim=-1)
        if self.vocab_size is not None and logits.shape[-1] > self.vocab_size:
            logits = logits[:, :self.vocab_size].contiguous()
        if bitmask is not None:
            logits = logits.clone() if not logits.is_contiguous() else logits
            S.apply_token_bitmask(logits, bitmask)
        if min_p is None:
            min_p = torch.zeros_like(temperature)
        return ops.sample(logits, temperature, top_k, top_p, seeds, offsets, min_p=min_p,
                          out_logprob=out_logprob)


def rejection_sampler(target_tokens: torch.Tensor, draft_tokens: torch.Tensor,
                      num_drafts: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy verification on the device, batched: ``target_tokens [B, k + 1]`` (the target's
    choice after each position), ``draft_tokens [B, k]`` -> ``[B, k + 1]`` accepted tokens with
    -1 padding: drafts are kept while they equal the target's token, the first mismatch is
    replaced by the target's token, and a fully accepted row gets the bonus token.
    ``num_drafts [B]`` limits rows with fewer than k drafts."""
    B, k1 = target_tokens.shape
    k = k1 - 1
    match = (draft_tokens == target_tokens[:, :k])
    if num_drafts is not None:
        valid = torch.arange(k, device=draft_tokens.device)[None, :] < num_drafts[:, None]
        match = match & valid
    # number of leading matches
    n_acc = torch.cumprod(match.to(torch.int32), dim=1).sum(dim=1)
    out = torch.full((B, k1), -1, dtype=target_tokens.dtype, device=target_tokens.device)
    pos = torch.arange(k1, device=target_tokens.device)[None, :]
    keep = pos <= n_acc[:, None]
    out[keep] = target_tokens[keep]
    return out
