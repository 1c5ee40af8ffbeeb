"""Fused tensor-parallel collectives over symmetric NVLink peer memory (decode path).

``TPFusedComm`` owns, on every rank of a TP group, one symmetric allocation laid out as

    [ receive slots: 2 x world x max_rows x H bf16 | flags: 2 x max_rows x world u32 ]

mapped on every peer through CUDA IPC.  ``allreduce_norm`` finishes a row-parallel
projection (``o_proj`` / ``down_proj``) whose local split-K GEMM accumulated fp32 partial sums:
one kernel pushes each bf16 partial row into every peer's receive slot, signals a per-row
flag, waits for the peers' rows, and computes ``residual += sum(partials)`` in rank order
followed by RMSNorm, so every rank ends with the same normalized activation for the next
column-parallel GEMM.  This is the B200 replacement of ``RowParallelLinear`` + all-reduce +
residual + norm (reference: vllm_neuron/nn/rpl.py:23-154; all-reduce sites
vllm_neuron/model/llama3/model.py:989,1113).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext
from .comm import GroupComm


class TPFusedComm:
    def __init__(self, tp: GroupComm, hidden: int, max_rows: int, device: torch.device,
                 cpu_group=None):
        assert 1 < tp.world <= 8
        self.tp = tp
        self.W, self.rank = tp.world, tp.rank
        self.H = hidden
        self.max_rows = max_rows
        self.device = device
        slot_bytes = 2 * self.W * max_rows * hidden * 2
        self.off_flags = _align(slot_bytes)
        total = self.off_flags + _align(2 * max_rows * self.W * 4)
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
        self.recv_ptrs = list(self.peers)
        self.flag_ptrs = [p + self.off_flags for p in self.peers]
        self.state = torch.zeros(2, dtype=torch.int64, device=device)
        dist.barrier(group=cpu_group)

    def allreduce_norm(self, acc: torch.Tensor, residual: torch.Tensor, norm_w: torch.Tensor,
                       eps: float, out: torch.Tensor) -> torch.Tensor:
        """``residual += all_reduce(acc)``; ``out = rmsnorm(residual) * norm_w``; clears ``acc``."""
        ext().tp_allreduce_norm(acc, self.recv_ptrs, self.flag_ptrs, self.state, residual, norm_w,
                                out, eps, self.rank, self.max_rows)
        return out

    def close(self):
        for p in self._opened:
            try:
                ext().symm_close(p)
            except Exception:
                pass
        self._opened = []


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a
