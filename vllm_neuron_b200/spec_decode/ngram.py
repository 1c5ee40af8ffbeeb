"""N-gram (prompt lookup) proposer: the draft continues the most recent earlier occurrence of
the context's last n tokens (n from ``max_n`` down to ``min_n``)."""
from __future__ import annotations

import numpy as np


class NgramProposer:
    def __init__(self, num_speculative_tokens: int, min_n: int = 1, max_n: int = 4,
                 max_context: int = 4096):
        self.k = num_speculative_tokens
        self.min_n, self.max_n = min_n, max_n
        self.max_context = max_context

    def propose_one(self, tokens: list[int]) -> list[int]:
        ctx = np.asarray(tokens[-self.max_context:], dtype=np.int64)
        L = len(ctx)
        for n in range(min(self.max_n, L - 1), self.min_n - 1, -1):
            pat = ctx[L - n:]
            # candidate starts whose n-gram matches, excluding the suffix itself
            win = np.lib.stride_tricks.sliding_window_view(ctx[:L - 1], n)
            hits = np.nonzero((win == pat).all(axis=1))[0]
            if len(hits):
                s = int(hits[-1]) + n
                draft = ctx[s:s + self.k].tolist()
                if draft:
                    return draft
        return []

    def propose(self, requests) -> dict[str, list[int]]:
        return {r.request_id: self.propose_one(r.all_token_ids()) for r in requests}
