"""Verification of draft tokens against the target model's logits.

For a request whose step computed the logits rows ``l_0 .. l_k`` (row j scores the token after
position j of ``[last, d_1, .., d_k]``):

* greedy: accept ``d_{j+1}`` while it equals ``argmax l_j``; the first mismatch is replaced by
  ``argmax l_j``; if all k are accepted the bonus token is ``argmax l_k``;
* random (temperature T): the drafts of these proposers are deterministic (one-hot draft
  distribution q), so ``d_{j+1}`` is accepted with probability ``p_j(d_{j+1})`` where
  ``p_j = softmax(l_j / T)``; on rejection the token is drawn from ``p_j`` with ``d_{j+1}``
  removed and renormalised (the residual ``max(0, p - q)`` of Leviathan et al.), which keeps
  the output distribution exactly that of the target model.

Returns the accepted tokens per request (1..k+1 tokens).  Reference:
vllm_neuron/vllm/sample/rejection_sampler.py:19-596, nn/rejection_sampler.py:12.
"""
from __future__ import annotations

import torch


def rejection_sample(logits: torch.Tensor, drafts: list[list[int]], temperatures: list[float],
                     generators: list[torch.Generator | None] | None = None) -> list[list[int]]:
    """``logits [sum(len(d) + 1), V]`` rows grouped per request in order."""
    out = []
    row = 0
    greedy_rows = logits.argmax(-1).tolist()
    for i, d in enumerate(drafts):
        n = len(d) + 1
        t = temperatures[i]
        toks: list[int] = []
        if t is None or t <= 1e-5:
            for j in range(n):
                best = greedy_rows[row + j]
                if j < len(d) and d[j] == best:
                    toks.append(d[j])
                    continue
                toks.append(best)
                break
        else:
            g = generators[i] if generators else None
            probs = torch.softmax(logits[row:row + n].float() / t, dim=-1)
            for j in range(n):
                p = probs[j]
                if j < len(d):
                    u = torch.rand((), generator=g, device="cpu").item() if g is not None else torch.rand(()).item()
                    if u < p[d[j]].item():
                        toks.append(d[j])
                        continue
                    p = p.clone()
                    p[d[j]] = 0
                    p = p / p.sum().clamp_min(1e-20)
                toks.append(int(torch.multinomial(p.cpu(), 1, generator=g).item()))
                break
        out.append(toks)
        row += n
    return out


def rejection_sample_ref(target_argmax: list[list[int]], drafts: list[list[int]]) -> list[list[int]]:
    """Greedy oracle on precomputed per-row argmax lists (``len(d) + 1`` entries each)."""
    res = []
    for am, d in zip(target_argmax, drafts):
        toks = []
        for j in range(len(d) + 1):
            if j < len(d) and d[j] == am[j]:
                toks.append(d[j])
            else:
                toks.append(am[j])
                break
        res.append(toks)
    return res
