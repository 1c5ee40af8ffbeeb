"""Device-side expert-parallel token exchange over NVLink peer memory (csrc/comm/ep_fused.cu).

:class:`EPFusedExchange` is the CUDA counterpart of :class:`..parallel.all2all.All2AllManager`
for MoE layers whose EP ranks hold different tokens (data-parallel attention replicas, wide
EP).  Instead of a host count exchange and two NCCL all-to-all-v per direction, four kernels do
the exchange on the device:

* ``dispatch(x, ids, w)``: each token's row, its k expert ids (other ranks' experts masked to
  -1) and weights are stored once into every destination rank's receive buffer (one slot
  taken with a system-scope atomic per destination);
* ``recv()``: waits for every source, marks the unused receive rows, and returns fixed-size
  views ``(rows [rows_cap, H], ids [rows_cap, k], w [rows_cap, k])`` over this rank's buffer
  that the expert pipeline (align, grouped tcgen05 GEMMs, weighted combine) consumes directly;
* ``ret(y)``: stores each reduced row into its token owner's combine slot;
* ``combine(out)``: sums each token's slots over the ranks it was sent to, in rank order.

All sizes are static (``tokens_cap`` tokens per rank, ``world * tokens_cap`` receive rows) and
the call counter lives on the device, so an EP step can be captured in a CUDA graph.  Every rank
of the EP group must make the same sequence of calls (one per MoE layer per step; an idle
data-parallel replica runs a dummy step).  Reference: vllm_neuron/parallel/all2all.py:113-517
(dispatch / combine managers), functional/collectives/reduce_scatter_v.py:53-365,
functional/moe/permute_routed_tokens.py:26.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext
from .fused import _align


class EPFusedExchange:
    def __init__(self, group, rank: int, world: int, num_experts: int, k: int, hidden: int,
                 tokens_cap: int, device: torch.device, cpu_group=None):
        if num_experts % world:
            raise ValueError(f"{num_experts} experts are not divisible by the EP size {world}")
        if world > 8 or hidden % 8:
            raise ValueError("EP exchange: at most 8 ranks and a hidden size divisible by 8")
        self.rank, self.world, self.E, self.k, self.H = rank, world, num_experts, k, hidden
        self.e_local = num_experts // world
        self.e_start = rank * self.e_local
        self.tokens_cap = tokens_cap
        self.rows_cap = world * tokens_cap
        self.device = device
        R, T = self.rows_cap, tokens_cap
        offs, o = [], 0
        for nbytes in (4 * (1 + 2 * 8), 2 * R * hidden, 4 * R * k, 4 * R * k, 4 * R, 2 * T * world * hidden):
            offs.append(o)
            o = _align(o + nbytes)
        self.offs = offs
        with torch.cuda.device(device):
            ptr, handle = ext().symm_alloc(o)
        self._local = ptr
        handles = [None] * dist.get_world_size()
        dist.all_gather_object(handles, (dist.get_rank(), handle), group=cpu_group)
        by_rank = {r: h for r, h in handles}
        ranks = dist.get_process_group_ranks(group) if group is not None else list(range(world))
        self.peers, self._opened = [], []
        with torch.cuda.device(device):
            for gr in ranks:
                if gr == dist.get_rank():
                    self.peers.append(ptr)
                else:
                    q = ext().symm_open(by_rank[gr])
                    self.peers.append(q)
                    self._opened.append(q)
        dev = device.index if device.index is not None else torch.cuda.current_device()
        view = lambda off, shape, dt: ext().tensor_from_ptr(ptr + off, shape, dt, dev)  # noqa: E731
        self.recv_rows = view(offs[1], [R, hidden], torch.bfloat16)
        self.recv_ids = view(offs[2], [R, k], torch.int32)
        self.recv_w = view(offs[3], [R, k], torch.float32)
        self.recv_count = torch.zeros(1, dtype=torch.int32, device=device)
        self.ctas_done = torch.zeros(1, dtype=torch.int32, device=device)
        self.state = torch.zeros(1, dtype=torch.int64, device=device)
        self.calls = 0
        dist.barrier(group=cpu_group)

    def _dims(self, T: int) -> list[int]:
        return [self.rank, self.world, self.H, self.k, self.E, self.e_local, self.tokens_cap,
                self.rows_cap, T]

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor):
        T = x.shape[0]
        if T > self.tokens_cap:
            raise ValueError(f"{T} tokens exceed the EP exchange capacity {self.tokens_cap}")
        self._ids, self._T = ids.to(torch.int32).contiguous(), T
        ext().ep_exchange(0, self.peers, self.offs, self._dims(T), x, self._ids, w.float().contiguous(),
                          None, None, self.recv_count, self.ctas_done, self.state)

    def recv(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        ext().ep_exchange(1, self.peers, self.offs, self._dims(self._T), None, None, None, None, None,
                          self.recv_count, self.ctas_done, self.state)
        return self.recv_rows, self.recv_ids, self.recv_w

    def ret(self, y: torch.Tensor):
        ext().ep_exchange(2, self.peers, self.offs, self._dims(self._T), None, None, None, None, y,
                          self.recv_count, self.ctas_done, self.state)

    def combine(self, out: torch.Tensor) -> torch.Tensor:
        ext().ep_exchange(3, self.peers, self.offs, self._dims(self._T), None, self._ids, None, out, None,
                          self.recv_count, self.ctas_done, self.state)
        self.calls += 1
        return out

    def close(self):
        for q in self._opened:
            try:
                ext().symm_close(q)
            except Exception:
                pass
        self._opened = []
