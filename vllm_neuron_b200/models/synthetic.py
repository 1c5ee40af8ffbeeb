"""Synthetic test model: exercises the KV-cache plumbing without any learned weights.

Every forward writes, for each token at position p, K = f(p, layer, head, d) and
V = -f(p, layer, head, d) into the paged cache at the token's slot; for every sampling row it
then reads back all KV positions of its sequence through the block table and emits status
token ``5`` when every value matches (``6`` otherwise).  A block-table, slot-mapping,
prefix-cache or preemption bug therefore shows up as a ``6`` in the output.

Reference: vllm_neuron/model/synthetic/synthetic.py (deterministic KV fill on prefill, exact
KV verify on decode, status tokens) and its sharding helpers.
"""
from __future__ import annotations

import torch

from ..config import ModelArchConfig
from ..parallel.comm import SINGLE, GroupComm

STATUS_OK = 5
STATUS_KV_MISMATCH = 6


class SyntheticForCausalLM(torch.nn.Module):
    supports_prefix_caching = True
    supports_cuda_graphs = False  # host-side verification loop

    def __init__(self, cfg: ModelArchConfig, tp: GroupComm = SINGLE, device="cuda", dtype=torch.bfloat16,
                 max_tokens: int = 8192, max_decode_tokens: int = 128, max_seqs: int = 256,
                 block_size: int = 16):
        super().__init__()
        self.cfg = cfg
        self.tp = tp
        self.device = torch.device(device)
        self.dtype = dtype
        self.Hkv = max(1, cfg.num_kv_heads // tp.world)
        self.Hq = self.Hkv
        self.D = cfg.head_dim
        self.H = cfg.hidden_size
        self.V = cfg.vocab_size
        self.block_size = block_size
        self.max_decode_tokens = max_decode_tokens
        self.max_tokens = max_tokens
        self.attn_splits_max = 1
        self.tp_fused = None
        self.kv_caches: list = []
        self.head_base = tp.rank * self.Hkv

    @property
    def num_kv_layers(self) -> int:
        return self.cfg.num_layers

    def kv_cache_shape(self, num_blocks: int):
        return (num_blocks, self.Hkv, self.block_size, self.D)

    def kv_bytes_per_block(self) -> int:
        return 2 * self.num_kv_layers * self.Hkv * self.block_size * self.D * torch.finfo(self.dtype).bits // 8

    def bind_kv_cache(self, kv_caches):
        self.kv_caches = kv_caches

    def init_random(self, seed: int = 0, std: float = 0.02):
        pass

    def load_hf_state_dict(self, get_tensor, names):
        pass

    def enable_fused_comm(self, cpu_group=None, fused_sp: bool = False):
        pass

    def _expected(self, pos: torch.Tensor, layer: int) -> torch.Tensor:
        """f(p, l, h, d) in [-1, 1), exactly representable in bf16 (multiples of 1/128)."""
        h = torch.arange(self.Hkv, device=pos.device) + self.head_base
        d = torch.arange(self.D, device=pos.device)
        v = (pos[:, None, None] * 31 + layer * 17 + h[None, :, None] * 7 + d[None, None, :]) % 256
        return (v.float() - 128.0) / 128.0

    @torch.no_grad()
    def forward(self, b) -> torch.Tensor:
        T = b.num_tokens
        pos = b.positions[:T].long()
        slots = b.slot_mapping[:T].long()
        bs = self.block_size
        ok_tok = slots >= 0
        for l, (kc, vc) in enumerate(self.kv_caches):
            e = self._expected(pos, l).to(kc.dtype)
            s = slots[ok_tok]
            kc.view(-1, self.Hkv, bs, self.D)  # layout check
            kc[s // bs, :, s % bs] = e[ok_tok]
            vc[s // bs, :, s % bs] = -e[ok_tok]
        # verify every sequence that samples
        B = b.seq_lens.shape[0]
        q_start = b.q_start.long()
        seq_lens = b.seq_lens.long()
        status = torch.full((B,), STATUS_OK, dtype=torch.long, device=pos.device)
        for i in range(B):
            L = int(seq_lens[i])
            p = torch.arange(L, device=pos.device)
            blk = b.block_tables[i, p // bs].long()
            for l, (kc, vc) in enumerate(self.kv_caches):
                e = self._expected(p, l)
                k = kc[blk, :, p % bs].float()
                v = vc[blk, :, p % bs].float()
                if not (torch.equal(k, e) and torch.equal(v, -e)):
                    status[i] = STATUS_KV_MISMATCH
                    break
        idx = b.logits_indices.long()
        seq_of = torch.searchsorted(q_start[1:], idx, right=True)
        logits = torch.full((idx.shape[0], self.V), -1e4, dtype=self.dtype, device=pos.device)
        logits[torch.arange(idx.shape[0], device=pos.device), status[seq_of]] = 0.0
        return logits
