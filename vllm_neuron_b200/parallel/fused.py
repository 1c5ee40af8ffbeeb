"""Fused tensor-parallel collectives over symmetric NVLink peer memory: the decode all-reduce
(``TPFusedComm``) and the sequence-parallel prefill all-gather / reduce-scatter fused into the
GEMMs and the RMSNorm (``SPFusedComm``).

``TPFusedComm`` owns, on every rank of a TP group, one symmetric allocation laid out as

    [ receive slots: 3 x world x max_rows x H bf16 | flags: 2 x max_rows x world u32 ]

mapped on every peer through CUDA IPC.  ``allreduce_norm`` finishes a row-parallel
projection (``o_proj`` / ``down_proj``) whose local split-K GEMM accumulated fp32 partial sums:
one kernel stores each bf16 partial row into every rank's receive slot and computes
``residual += sum(partials)`` in rank order followed by RMSNorm, so every rank ends with the same
normalized activation for the next column-parallel GEMM.  The slots hold the bf16 sentinel
0x8000 (negative zero) where no data has arrived, so the reader polls the data itself -- no
fence and no flag round trip per call (three slot sets rotate; each call resets the previous
call's set).  ``algo = 1`` selects the older form (per-row flags raised after a system-scope
fence, two slot sets), kept for comparison; one object must keep one form.  This is the B200
replacement of ``RowParallelLinear`` + all-reduce + residual + norm (reference:
vllm_neuron/nn/rpl.py:23-154; all-reduce sites vllm_neuron/model/llama3/model.py:989,1113).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext
from .comm import GroupComm


class TPFusedComm:
    def __init__(self, tp: GroupComm, hidden: int, max_rows: int, device: torch.device,
                 cpu_group=None, algo: int = 0):
        assert 1 < tp.world <= 8 and algo in (0, 1)
        self.tp = tp
        self.W, self.rank = tp.world, tp.rank
        self.H = hidden
        self.max_rows = max_rows
        self.device = device
        slot_bytes = 3 * self.W * max_rows * hidden * 2
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
        # [0] calls completed, [1] CTAs finished in the running call, [2] rows of the last call
        self.state = torch.zeros(4, dtype=torch.int64, device=device)
        self.algo = algo
        if algo == 0:  # every slot starts as the "not arrived" sentinel
            dev = device.index if device.index is not None else torch.cuda.current_device()
            ext().tensor_from_ptr(ptr, [slot_bytes // 2], torch.bfloat16, dev).fill_(-0.0)
            torch.cuda.synchronize(device)
        dist.barrier(group=cpu_group)

    def allreduce_norm(self, acc: torch.Tensor, residual: torch.Tensor, norm_w: torch.Tensor,
                       eps: float, out: torch.Tensor) -> torch.Tensor:
        """``residual += all_reduce(acc)``; ``out = rmsnorm(residual) * norm_w``; clears ``acc``."""
        ext().tp_allreduce_norm(acc, self.recv_ptrs, self.flag_ptrs, self.state, residual, norm_w, out,
                                eps, self.rank, self.max_rows, self.algo)
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


def _exchange_handles(tp: GroupComm, ptr: int, handle, device, cpu_group) -> tuple[list[int], list[int]]:
    handles = [None] * dist.get_world_size()
    dist.all_gather_object(handles, (dist.get_rank(), handle), group=cpu_group)
    by_rank = {r: h for r, h in handles}
    peers, opened = [], []
    with torch.cuda.device(device):
        for gr in tp.ranks:
            if gr == dist.get_rank():
                peers.append(ptr)
            else:
                q = ext().symm_open(by_rank[gr])
                peers.append(q)
                opened.append(q)
    return peers, opened


class SPFusedComm:
    """Sequence-parallel prefill with the collectives fused into the kernels.

    Each rank owns ``Tl = Tg / W`` consecutive token rows of the residual stream.  One symmetric
    allocation per rank, mapped on every peer:

        [ x: 2 x Tg_max x H bf16 | slots: 2 x W x Tl_max x H bf16 | rs_ctr: W u32 | ag_ctr: W u32 ]

    * ``gemm_rs`` (o_proj / down_proj): one GEMM over all tokens whose epilogue stores each
      output row into the owning rank's ``slots[parity][this rank]`` over NVLink and raises the
      owner's ``rs_ctr[this rank]`` per tile (reduce-scatter fused into the GEMM);
    * ``norm_push``: waits for every source's tiles, sums them in rank order with the residual,
      RMSNorm, and pushes the normalized rows into every rank's ``x[parity]`` (all-gather fused
      into the norm), raising each rank's ``ag_ctr[this rank]`` per CTA;
    * ``gemm_ag`` (qkv / gate_up): the GEMM over ``x`` whose TMA producer waits on
      ``ag_ctr[r]`` before the first load of rank r's rows, so local rows start at once.

    Counters only grow; this object tracks the cumulative targets (all ranks run the same
    sequence of calls with the same sizes).  Reference: SP prefill,
    vllm_neuron/model/llama3/model.py:527-532,813-815,1096-1111."""

    def __init__(self, tp: GroupComm, hidden: int, max_tokens: int, device: torch.device, cpu_group=None):
        assert 1 < tp.world <= 8
        self.tp = tp
        self.W, self.rank, self.H = tp.world, tp.rank, hidden
        self.Tg_max = -(-max_tokens // self.W) * self.W
        self.Tl_max = self.Tg_max // self.W
        self.x_bytes = self.Tg_max * hidden * 2
        self.off_slots = _align(2 * self.x_bytes)
        self.slot_bytes = self.Tl_max * hidden * 2
        self.off_ctr = _align(self.off_slots + 2 * self.W * self.slot_bytes)
        total = self.off_ctr + _align(2 * self.W * 4)
        self.device = device
        with torch.cuda.device(device):
            ptr, handle = ext().symm_alloc(total)
        self._local = ptr
        self.peers, self._opened = _exchange_handles(tp, ptr, handle, device, cpu_group)
        self.ag_calls = 0
        self.rs_calls = 0
        self.ag_target = [0] * self.W   # cumulative CTAs pushed to this rank by each source
        self.rs_target = 0              # cumulative tiles each source stored into this rank
        self.forwards = 0
        dist.barrier(group=cpu_group)

    # ---- addresses
    def _x(self, r: int, par: int) -> int:
        return self.peers[r] + par * self.x_bytes

    def _slot(self, r: int, par: int, src: int) -> int:
        return self.peers[r] + self.off_slots + (par * self.W + src) * self.slot_bytes

    def _rs_ctr(self, r: int, src: int) -> int:
        return self.peers[r] + self.off_ctr + 4 * src

    def _ag_ctr(self, r: int, src: int) -> int:
        return self.peers[r] + self.off_ctr + 4 * (self.W + src)

    def x_view(self, par: int, rows: int) -> torch.Tensor:
        return ext().tensor_from_ptr(self._x(self.rank, par), [rows, self.H], torch.bfloat16,
                                     self.device.index if self.device.index is not None else torch.cuda.current_device())

    # ---- fused collectives
    def norm_push(self, residual: torch.Tensor, w: torch.Tensor, eps: float, reduce: bool) -> torch.Tensor:
        """``residual += sum of the sources' slots`` (``reduce``), RMSNorm, all-gather push;
        returns this rank's view ``[Tg, H]`` of the gathered normalized rows (complete once the
        consumer GEMM's waits, or :meth:`wait_gathered`, pass)."""
        Tl = residual.shape[0]
        assert Tl <= self.Tl_max
        par = self.ag_calls % 2
        self.ag_calls += 1
        rs_par = (self.rs_calls - 1) % 2
        ext().sp_norm_push(self._slot(self.rank, rs_par, 0), self.Tl_max * self.H, self.W if reduce else 0,
                           self._rs_ctr(self.rank, 0), self.rs_target, residual, w, eps,
                           [self._x(r, par) + self.rank * Tl * self.H * 2 for r in range(self.W)],
                           [self._ag_ctr(r, self.rank) for r in range(self.W)])
        self.ag_target = [t + Tl for t in self.ag_target]
        self._Tl = Tl
        return self.x_view(par, Tl * self.W)

    @staticmethod
    def _w(w):
        """(weight tensor, block scales or None): bf16 weights or block-scaled FP8 ones."""
        from ..ops.linear import BlockFP8Weight

        return (w.q, w.scales) if isinstance(w, BlockFP8Weight) else (w, None)

    def gemm_ag(self, x: torch.Tensor, w, out: torch.Tensor, epi: int, bn: int) -> torch.Tensor:
        """GEMM over the all-gathered rows ``x`` (a view from :meth:`norm_push`)."""
        wt, sc = self._w(w)
        ext().gemm_sp(x, wt, out, epi, bn, self._ag_ctr(self.rank, 0), self.ag_target, self._Tl, [], [], 0, sc)
        return out

    def gemm_rs(self, a: torch.Tensor, w: torch.Tensor, bn: int) -> None:
        """Row-parallel GEMM of all ``Tg`` rows reduce-scattered into the owners' slots."""
        Tg, N = a.shape[0], w.shape[0]
        Tl = Tg // self.W
        par = self.rs_calls % 2
        self.rs_calls += 1
        carrier = self.x_view(0, 1)  # row stride H for the slot stores
        wt, sc = self._w(w)
        ext().gemm_sp(a, wt, carrier, 5, bn, 0, [], 0,
                      [self._slot(r, par, self.rank) for r in range(self.W)],
                      [self._rs_ctr(r, self.rank) for r in range(self.W)], Tl, sc)
        nb = -(-N // bn)
        lo, hi = (self.rank * Tl) // 128, ((self.rank + 1) * Tl - 1) // 128
        self.rs_target += (hi - lo + 1) * nb

    def wait_gathered(self):
        """Order the following kernels after every source's push of the last ``norm_push``."""
        ext().sp_wait(self._ag_ctr(self.rank, 0), self.ag_target)

    def close(self):
        for p in self._opened:
            try:
                ext().symm_close(p)
            except Exception:
                pass
        self._opened = []
