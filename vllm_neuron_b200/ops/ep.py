"""Expert-parallel token exchange: dispatch metadata, routed-token packing and the combine-side
reduction, for MoE layers whose experts are sharded over an EP group of ranks that each hold
different tokens (data-parallel attention, wide EP).

Layout.  Rank ``d`` of the EP group owns experts ``[d * e_local, (d + 1) * e_local)``.  A
token is sent once to every rank that owns at least one of its top-k experts (tokens whose
experts share a rank are deduplicated), as one row of the hidden state plus an affinity row of
``e_local`` weights (zero for that rank's experts the token did not select).  The receiving rank
runs its experts on the rows it received and reduces each row over its selected experts with
those weights; the partial rows travel back and :func:`topk_reduce` sums the partials of each
token.  Rows are ordered by destination rank and then by token, so one variable-size
all-to-all per direction moves them.

Reference: vllm_neuron/functional/moe/build_all2all_dispatch_metadata.py:24 (send counts from
expert indices, deduplicated per rank), permute_routed_tokens.py:26 (packing rows sorted by
destination), build_all2all_combine_metadata.py:13 (combine metadata from the saved counts),
topk_reduce.py:28 (sum of scattered rows by token) and pack_tokens.py:19.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class DispatchPlan:
    """Host-known sizes and device index tensors of one exchange."""

    send_counts: list[int]          # rows to each destination rank
    recv_counts: list[int]          # rows from each source rank (filled by the exchange)
    token_of_row: torch.Tensor      # [rows] int64: source token of each sent row
    dest_of_row: torch.Tensor       # [rows] int64
    num_tokens: int


def build_dispatch_metadata(ids: torch.Tensor, e_local: int, world: int) -> tuple[DispatchPlan, torch.Tensor]:
    """From ``ids [T, k]`` (global expert ids; negative = no expert) build the deduplicated
    send plan and ``hit [T, world]`` (token t goes to rank d)."""
    T = ids.shape[0]
    dest = torch.div(ids.long().clamp(min=0), e_local, rounding_mode="floor")
    valid = ids >= 0
    hit = torch.zeros(T, world, dtype=torch.bool, device=ids.device)
    hit.scatter_(1, dest.masked_fill(~valid, 0), valid)
    # rows ordered by destination, then token
    d_idx, t_idx = torch.nonzero(hit.t(), as_tuple=True)
    send_counts = torch.bincount(d_idx, minlength=world)
    plan = DispatchPlan(send_counts=[int(c) for c in send_counts.tolist()], recv_counts=[0] * world,
                        token_of_row=t_idx, dest_of_row=d_idx, num_tokens=T)
    return plan, hit


def permute_routed_tokens(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                          plan: DispatchPlan, e_local: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Send buffers of ``plan``: ``rows [R, H]`` (hidden of each row's token) and
    ``aff [R, e_local]`` fp32 (the token's weights for the destination's experts)."""
    t = plan.token_of_row
    d = plan.dest_of_row
    rows = x.index_select(0, t)
    R = t.numel()
    aff = torch.zeros(R, e_local, dtype=torch.float32, device=x.device)
    if R:
        ids_r = ids.long().index_select(0, t)                       # [R, k]
        w_r = weights.float().index_select(0, t)                    # [R, k]
        local = ids_r - d[:, None] * e_local
        sel = (ids_r >= 0) & (local >= 0) & (local < e_local)
        aff.scatter_add_(1, local.clamp(0, e_local - 1), torch.where(sel, w_r, torch.zeros_like(w_r)))
    return rows, aff


def local_routing(aff: torch.Tensor, e_start: int, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Received affinity rows -> ``(ids [R, k], weights [R, k])`` over this rank's experts in the
    layout the expert kernels take (unused slots get an expert id outside the local range)."""
    R, e_local = aff.shape
    kk = min(k, e_local)
    w, j = torch.topk(aff, kk, dim=1)
    ids = torch.where(w > 0, j + e_start, torch.full_like(j, -1)).to(torch.int32)
    w = torch.where(w > 0, w, torch.zeros_like(w))
    if kk < k:
        pad = k - kk
        ids = torch.cat([ids, torch.full((R, pad), -1, dtype=torch.int32, device=aff.device)], 1)
        w = torch.cat([w, torch.zeros(R, pad, dtype=w.dtype, device=aff.device)], 1)
    return ids.contiguous(), w.float().contiguous()


def topk_reduce(partials: torch.Tensor, plan: DispatchPlan, out: torch.Tensor | None = None) -> torch.Tensor:
    """Sum the returned partial rows of each token: ``out[t] = sum_{rows r of t} partials[r]``."""
    H = partials.shape[1]
    acc = torch.zeros(plan.num_tokens, H, dtype=torch.float32, device=partials.device)
    if partials.shape[0]:
        acc.index_add_(0, plan.token_of_row, partials.float())
    if out is None:
        return acc.to(partials.dtype)
    out.copy_(acc.to(out.dtype))
    return out


def pack_tokens(index: torch.Tensor) -> torch.Tensor:
    """Positions of the rows with a non-negative index, in order (moves them to the front)."""
    return torch.nonzero(index >= 0, as_tuple=True)[0]
