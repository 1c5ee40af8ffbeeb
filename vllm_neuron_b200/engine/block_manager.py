"""Paged KV block allocator with automatic prefix caching.

Block 0 is the reserved null block (padding and unused block-table entries point at it, as
in the reference: vllm_neuron/vllm/worker/neuron_model_runner.py:94-110).  Full blocks of a
request are content-addressed by a chained hash of their token ids; a later request with
the same prefix reuses them (reference: prefix caching through upstream vLLM block hashing,
docs/design/vllm/prefix-caching.md).  Freed cached blocks stay reusable until evicted in LRU
order.
"""
from __future__ import annotations

from collections import OrderedDict


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, enable_prefix_caching: bool = False):
        assert num_blocks >= 2
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.enable_prefix_caching = enable_prefix_caching
        self.free: list[int] = list(range(num_blocks - 1, 0, -1))  # pop() -> lowest id first
        self.ref = [0] * num_blocks
        self.block_hash: dict[int, int] = {}        # block id -> hash (full cached blocks)
        self.hash_to_block: dict[int, int] = {}     # hash -> block id
        self.evictable: OrderedDict[int, None] = OrderedDict()  # ref==0 cached blocks, LRU
        self.req_hashes: dict[str, list[int]] = {}

    # ------------------------------------------------------------------ accounting
    @property
    def num_free_blocks(self) -> int:
        return len(self.free) + len(self.evictable)

    def usage(self) -> float:
        return 1.0 - self.num_free_blocks / (self.num_blocks - 1)

    def blocks_needed(self, req, num_tokens: int) -> int:
        need = (num_tokens + self.block_size - 1) // self.block_size
        return max(0, need - len(req.block_ids))

    # ------------------------------------------------------------------ hashing
    def _chain_hashes(self, token_ids: list[int], n_full: int) -> list[int]:
        hs, h, bs = [], 0, self.block_size
        for i in range(n_full):
            h = hash((h, tuple(token_ids[i * bs:(i + 1) * bs])))
            hs.append(h)
        return hs

    def match_prefix(self, req) -> int:
        """Attach cached blocks for the longest cached prefix; returns #tokens covered."""
        if (not self.enable_prefix_caching or req.block_ids or getattr(req, "prompt_embeds", None) is not None
                or getattr(req, "mm", None) is not None):
            return 0  # prompt-embedding requests have no token ids to hash
        toks = req.prompt_token_ids
        # Keep at least one token to compute so the request produces logits.
        n_full = (len(toks) - 1) // self.block_size
        hashes = self._chain_hashes(toks, n_full)
        got = []
        for h in hashes:
            b = self.hash_to_block.get(h)
            if b is None:
                break
            got.append(b)
        for b in got:
            if self.ref[b] == 0:
                self.evictable.pop(b, None)
            self.ref[b] += 1
        req.block_ids.extend(got)
        self.req_hashes[req.request_id] = hashes[:len(got)]
        return len(got) * self.block_size

    # ------------------------------------------------------------------ alloc / free
    def _take(self) -> int | None:
        if self.free:
            return self.free.pop()
        if self.evictable:
            b, _ = self.evictable.popitem(last=False)
            h = self.block_hash.pop(b, None)
            if h is not None and self.hash_to_block.get(h) == b:
                del self.hash_to_block[h]
            return b
        return None

    def allocate(self, req, num_tokens: int) -> bool:
        """Ensure ``req`` has blocks for ``num_tokens`` tokens.  All-or-nothing."""
        need = self.blocks_needed(req, num_tokens)
        if need > self.num_free_blocks:
            return False
        for _ in range(need):
            b = self._take()
            self.ref[b] = 1
            req.block_ids.append(b)
        return True

    def commit_full_blocks(self, req):
        """Register the request's newly completed full blocks in the prefix cache."""
        if (not self.enable_prefix_caching or getattr(req, "prompt_embeds", None) is not None
                or getattr(req, "mm", None) is not None):
            return
        n_full = min(req.num_computed_tokens, req.num_tokens) // self.block_size
        hs = self.req_hashes.setdefault(req.request_id, [])
        if n_full <= len(hs):
            return
        toks = req.all_token_ids()
        h = hs[-1] if hs else 0
        for i in range(len(hs), n_full):
            h = hash((h, tuple(toks[i * self.block_size:(i + 1) * self.block_size])))
            hs.append(h)
            b = req.block_ids[i]
            if h not in self.hash_to_block:
                self.hash_to_block[h] = b
                self.block_hash[b] = h

    def free_request(self, req):
        for b in reversed(req.block_ids):
            self.ref[b] -= 1
            if self.ref[b] == 0:
                if b in self.block_hash:
                    self.evictable[b] = None
                else:
                    self.free.append(b)
        req.block_ids = []
        self.req_hashes.pop(req.request_id, None)

    def reset_prefix_cache(self):
        for b in list(self.evictable):
            self.block_hash.pop(b, None)
            self.free.append(b)
        self.evictable.clear()
        self.hash_to_block = {h: b for b, h in self.block_hash.items()}
