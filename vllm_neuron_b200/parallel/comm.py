"""Device collectives of a tensor-parallel group.

``GroupComm`` wraps one ``torch.distributed`` process group (NCCL over NVLink on B200,
gloo on CPU) with the in-place collectives the models use.  A world of one is a no-op.
The fused GEMM+collective kernels (``vllm_neuron_b200.parallel.fused``) replace these
calls on the hot paths when symmetric peer buffers are available; this class is the
baseline path and the fallback.

Reference: the GroupCoordinator-based collectives of vllm_neuron/parallel/
neuron_parallel_state.py and the call-site census of the models (e.g.
vllm_neuron/model/llama3/model.py:532,815,989,1098,1111).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class GroupComm:
    def __init__(self, group: dist.ProcessGroup | None = None, ranks: list[int] | None = None):
        self.group = group
        if group is None or not dist.is_initialized():
            self.rank, self.world = 0, 1
            self.ranks = [0]
        else:
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
            self.ranks = ranks if ranks is not None else list(range(self.world))
        self.is_gloo = group is not None and dist.is_initialized() and dist.get_backend(group) == "gloo"

    @property
    def is_single(self) -> bool:
        return self.world == 1

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather(self, t: torch.Tensor, dim: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        if self.world == 1:
            return t
        t = t.contiguous()
        if self.is_gloo:
            parts = [torch.empty_like(t) for _ in range(self.world)]
            dist.all_gather(parts, t, group=self.group)
            res = torch.cat(parts, dim=dim)
            if out is not None:
                out.copy_(res)
                return out
            return res
        if dim == 0:
            if out is None:
                out = torch.empty((t.shape[0] * self.world,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(out, t, group=self.group)
            return out
        g = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(g, t, group=self.group)
        parts = list(g.unbind(0))
        res = torch.cat(parts, dim=dim)
        if out is not None:
            out.copy_(res)
            return out
        return res

    def reduce_scatter(self, t: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Sum over ranks and keep this rank's 1/world slice of dim 0."""
        if self.world == 1:
            return t
        if out is None:
            out = torch.empty((t.shape[0] // self.world,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        if self.is_gloo:
            full = t.contiguous().clone()
            dist.all_reduce(full, group=self.group)
            out.copy_(full.chunk(self.world, 0)[self.rank])
            return out
        dist.reduce_scatter_tensor(out, t.contiguous(), group=self.group)
        return out

    def broadcast_(self, t: torch.Tensor, src: int = 0) -> torch.Tensor:
        if self.world > 1:
            dist.broadcast(t, src=self.ranks[src], group=self.group)
        return t

    def all_to_all(self, t: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if self.world == 1:
            return t
        if out is None:
            out = torch.empty_like(t)
        dist.all_to_all_single(out, t.contiguous(), group=self.group)
        return out


SINGLE = GroupComm(None)


class EmulatedRankComm(GroupComm):
    """One rank's share of a TP group of ``world`` ranks, run alone on one device.

    Shapes are sharded as for rank ``rank`` of ``world``, but every collective is local: an
    all-reduce keeps the local partial, an all-gather tiles the local shard.  The numbers it
    computes are not those of the real group; it exists so a single GPU can be profiled
    (ncu launch lists, per-kernel timings) with exactly one rank's kernel shapes.
    """

    def __init__(self, world: int, rank: int = 0):
        super().__init__(None)
        self.world, self.rank = world, rank
        self.ranks = list(range(world))

    def all_reduce_(self, t):
        return t

    def all_gather(self, t, dim: int = 0, out=None):
        res = torch.cat([t] * self.world, dim=dim)
        if out is not None:
            out.copy_(res)
            return out
        return res

    def reduce_scatter(self, t, out=None):
        part = t.chunk(self.world, 0)[self.rank]
        if out is not None:
            out.copy_(part)
            return out
        return part.contiguous()

    def broadcast_(self, t, src: int = 0):
        return t

    def all_to_all(self, t, out=None):
        if out is not None:
            out.copy_(t)
            return out
        return t.clone()
