"""Fused tensor-parallel collectives over symmetric NVLink peer memory (decode path).

``TPFusedComm`` owns, on every rank of a TP group, one symmetric allocation laid out as

    [ receive slots: world x max_rows_per_rank x H bf16 | activations x: max_tokens x H bf16 |
      slot-arrival counter u64 | row-arrival counter u64 ]

mapped on every peer through CUDA IPC.  ``rs_norm`` runs a row-parallel projection
(``o_proj`` / ``down_proj``) as

    gemm_tp_rs           split-K GEMM whose epilogue pushes each finished 128-column tile's
                         token rows (bf16) to the rank that owns them (reduce-scatter fused
                         into the GEMM, tile by tile)
    tp_norm_allgather    owner rank: sum the partials + residual, RMSNorm, store the row into
                         every rank's ``x`` (all-gather fused into the norm)

so every rank ends with the full normalized activation ``x`` for the next column-parallel
GEMM.  This is the B200 replacement of ``RowParallelLinear`` + all-reduce + residual + norm
(reference: vllm_neuron/nn/rpl.py:23-154; all-reduce sites vllm_neuron/model/llama3/
model.py:989,1113).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops import linear as L
from ..ops._ext import ext
from .comm import GroupComm


class TPFusedComm:
    def __init__(self, tp: GroupComm, hidden: int, max_tokens: int, device: torch.device,
                 cpu_group=None):
        assert tp.world > 1 and tp.world <= 8
        self.tp = tp
        self.W, self.rank = tp.world, tp.rank
        self.H = hidden
        self.max_tokens = max_tokens
        self.rpr_max = math.ceil(max_tokens / self.W)
        self.device = device
        slot_bytes = self.W * self.rpr_max * hidden * 2
        x_bytes = max_tokens * hidden * 2
        self.off_x = _align(slot_bytes)
        self.off_cnt = _align(self.off_x + x_bytes)
        total = self.off_cnt + 256
        with torch.cuda.device(device):
            ptr, handle = ext().symm_alloc(total)
        self._local = ptr
        handles = [None] * dist.get_world_size()
        dist.all_gather_object(handles, (dist.get_rank(), handle), group=cpu_group)
        by_rank = {r: h for r, h in handles}
        self.peers = []
        self._opened = []
        with torch.cuda.device(device):
            for gr in tp.ranks:
                if gr == dist.get_rank():
                    self.peers.append(ptr)
                else:
                    p = ext().symm_open(by_rank[gr])
                    self.peers.append(p)
                    self._opened.append(p)
        self.slot_ptrs = list(self.peers)
        self.x_ptrs = [p + self.off_x for p in self.peers]
        self.slot_arrive_ptrs = [p + self.off_cnt for p in self.peers]
        self.x_arrive_ptrs = [p + self.off_cnt + 8 for p in self.peers]
        dev_index = device.index if device.index is not None else torch.cuda.current_device()
        self.x = ext().tensor_from_ptr(self.x_ptrs[self.rank], [max_tokens, hidden], torch.bfloat16, dev_index)
        self.state = torch.zeros(2, dtype=torch.int64, device=device)
        self.tiles = math.ceil(hidden / 128)
        self.tile_count = torch.zeros(self.tiles, dtype=torch.int32, device=device)
        self.acc = torch.zeros(max_tokens, hidden, dtype=torch.float32, device=device)
        self.num_sms = torch.cuda.get_device_properties(device).multi_processor_count
        dist.barrier(group=cpu_group)

    def rs_norm(self, act: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                norm_w: torch.Tensor, eps: float) -> torch.Tensor:
        """``x = rmsnorm(residual += all_reduce(act @ w^T))`` for ``T = act.shape[0]`` rows;
        returns the full ``x [T, H]`` (this rank only updates the residual rows it owns)."""
        T, K = act.shape
        rpr = math.ceil(T / self.W)
        splits = L.pick_splits(self.H, K, self.num_sms)
        ext().gemm_tp_rs(w, act, self.acc[:T], splits, self.slot_ptrs, self.slot_arrive_ptrs,
                         self.tile_count, self.rank, rpr)
        ext().tp_norm_allgather(self.slot_ptrs[self.rank], self.slot_arrive_ptrs[self.rank],
                                self.x_ptrs, self.x_arrive_ptrs, self.state, residual, norm_w,
                                eps, self.rank, rpr, T, self.tiles)
        return self.x[:T]

    def close(self):
        for p in self._opened:
            try:
                ext().symm_close(p)
            except Exception:
                pass
        self._opened = []


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a
