"""On-device sampling (csrc/misc/sampling.cu) and its torch oracle.

Per-row parameters: temperature (<= 0: greedy), top_k (<= 0: off), top_p (>= 1: off),
min_p (<= 0: off), seed and step offset for the counter-based RNG.
Reference: vllm_neuron/functional/sampling.py:21, nn/sampler.py:13-169.
"""
from __future__ import annotations

import torch

from ._ext import ext


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
           top_p: torch.Tensor, seeds: torch.Tensor, offsets: torch.Tensor,
           min_p: torch.Tensor | None = None, out: torch.Tensor | None = None,
           out_logprob: torch.Tensor | None = None, vocab_offset: int = 0,
           row_slots: torch.Tensor | None = None, last_tok: torch.Tensor | None = None) -> torch.Tensor:
    """Sample one token per row.  With ``row_slots``, each row's token is also stored in
    ``last_tok[row_slots[row]]`` (the device-resident input of that request's next step)."""
    B = logits.shape[0]
    if out is None:
        out = torch.empty((B,), dtype=torch.int32, device=logits.device)
    if not logits.is_cuda:
        out.copy_(sample_ref(logits, temperature, top_k, top_p, seeds, offsets, min_p) + vocab_offset)
        if row_slots is not None:
            last_tok[row_slots.long()] = out
        return out
    ext().sample(logits, temperature, top_k, top_p, min_p, seeds, offsets, out, out_logprob,
                 vocab_offset, row_slots, last_tok)
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None,
           out_val: torch.Tensor | None = None, vocab_offset: int = 0) -> torch.Tensor:
    B = logits.shape[0]
    if out is None:
        out = torch.empty((B,), dtype=torch.int32, device=logits.device)
    if not logits.is_cuda:
        v, i = logits.float().max(dim=-1)
        out.copy_(i.to(torch.int32) + vocab_offset)
        if out_val is not None:
            out_val.copy_(v)
        return out
    ext().argmax(logits, out, out_val, vocab_offset)
    return out


def filter_mask_ref(x: torch.Tensor, k: int, p: float, min_p: float) -> torch.Tensor:
    """Boolean keep-mask of one row of temperature-scaled logits (fp32)."""
    V = x.numel()
    keep = torch.ones(V, dtype=torch.bool)
    if 0 < k < V:
        kth = torch.topk(x, k).values[-1]
        keep &= x >= kth
    if p < 1.0:
        m = x.max()
        e = torch.exp(x - m) * keep
        z = e.sum()
        vals, _ = torch.sort(x[keep], descending=True)
        ev = torch.exp(vals - m)
        cum = torch.cumsum(ev, 0)
        idx = int(torch.searchsorted(cum, p * z).clamp(max=len(vals) - 1))
        keep &= x >= vals[idx]
    if min_p > 0:
        keep &= x >= x.max() + torch.log(torch.tensor(min_p))
    return keep


def sample_ref(logits, temperature, top_k, top_p, seeds, offsets, min_p=None) -> torch.Tensor:
    """Greedy rows are exact; random rows draw with torch's generator (distributional oracle)."""
    B, V = logits.shape
    out = torch.empty(B, dtype=torch.int32)
    for b in range(B):
        t = float(temperature[b])
        row = logits[b].float().cpu()
        if t <= 0:
            out[b] = int(torch.argmax(row))
            continue
        x = row / t
        keep = filter_mask_ref(x, int(top_k[b]), float(top_p[b]),
                               float(min_p[b]) if min_p is not None else 0.0)
        probs = torch.softmax(x.masked_fill(~keep, float("-inf")), -1)
        g = torch.Generator().manual_seed((int(seeds[b]) * 1000003 + int(offsets[b])) & 0x7FFFFFFFFFFFFFFF)
        out[b] = int(torch.multinomial(probs, 1, generator=g))
    return out.to(logits.device)


def apply_token_bitmask(logits: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """``logits[r, i] = -inf`` where bit ``i`` of ``mask[r]`` (int32 words) is 0."""
    if not logits.is_cuda:
        V = logits.shape[1]
        bits = ((mask.to(torch.int64)[:, :, None] >> torch.arange(32)) & 1).reshape(mask.shape[0], -1)[:, :V]
        logits.masked_fill_(bits.to(logits.device) == 0, float("-inf"))
        return logits
    ext().apply_token_bitmask(logits, mask)
    return logits
