"""All-to-all expert-parallel exchange over a process group (wide EP).

:class:`All2AllManager` runs the two variable-size all-to-alls of an expert-parallel MoE layer
whose ranks hold different tokens: dispatch (rows of hidden states and expert affinities to the
ranks that own the selected experts) and combine (the experts' pre-reduced partial rows back to
the token owners).  The sizes are exchanged first with a fixed-size all-to-all of the counts, so
the row all-to-alls know their split sizes on the host; this path runs eagerly (outside CUDA
graphs), on NCCL for CUDA tensors and on gloo for CPU tensors.

Reference: ``NeuronAll2AllManager`` (vllm_neuron/parallel/all2all.py:33-641), mounted on the EP
group by ``NeuronDeviceCommunicator`` (parallel/neuron_communicator.py:13-51); the A2A-v with a
metadata pass (functional/collectives/all_to_all_v.py:21).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import ep as EP


class All2AllManager:
    def __init__(self, group, rank: int, world: int, num_experts: int):
        if num_experts % world:
            raise ValueError(f"{num_experts} experts are not divisible by the EP size {world}")
        self.group = group
        self.rank = rank
        self.world = world
        self.E = num_experts
        self.e_local = num_experts // world
        self.e_start = rank * self.e_local
        self.calls = 0

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
            return out
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        self.calls += 1
        return out

    def exchange_counts(self, plan: EP.DispatchPlan) -> None:
        dev = torch.device("cpu") if _cpu_group(self.group) else torch.device("cuda", torch.cuda.current_device())
        send = torch.tensor(plan.send_counts, dtype=torch.int64, device=dev)
        recv = torch.empty_like(send)
        self._a2a(recv, send, None, None)
        plan.recv_counts = [int(c) for c in recv.tolist()]

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor):
        """Returns ``(plan, recv_rows [R, H], recv_aff [R, e_local])``."""
        plan, _ = EP.build_dispatch_metadata(ids, self.e_local, self.world)
        self.exchange_counts(plan)
        rows, aff = EP.permute_routed_tokens(x, ids, weights, plan, self.e_local)
        R = sum(plan.recv_counts)
        recv_rows = torch.empty(R, x.shape[1], dtype=x.dtype, device=x.device)
        recv_aff = torch.empty(R, self.e_local, dtype=torch.float32, device=x.device)
        self._a2a(recv_rows, rows, plan.recv_counts, plan.send_counts)
        self._a2a(recv_aff, aff, plan.recv_counts, plan.send_counts)
        return plan, recv_rows, recv_aff

    def combine(self, partial_rows: torch.Tensor, plan: EP.DispatchPlan,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """Return the partial rows to their token owners and sum them per token."""
        back = torch.empty(sum(plan.send_counts), partial_rows.shape[1], dtype=partial_rows.dtype,
                           device=partial_rows.device)
        self._a2a(back, partial_rows.contiguous(), plan.send_counts, plan.recv_counts)
        return EP.topk_reduce(back, plan, out)


def _cpu_group(group) -> bool:
    try:
        return dist.get_backend(group) == "gloo"
    except Exception:
        return True
