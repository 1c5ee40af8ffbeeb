"""Mixture-of-experts ops (csrc/moe/moe.cu + the grouped mode of csrc/gemm/gemm_sm100.cu) and
their fp32 torch oracles.

Pipeline of one MoE block for ``x [T, H]`` on the experts ``[e_start, e_start + e_local)`` that
this rank holds (all experts without expert parallelism):

    logits = x @ router_w^T                        tcgen05 GEMM (bf16)
    ids, w = route(logits + router_b)              top-k per token (csrc moe_route)
    plan   = align(ids)                            expert-contiguous rows + tile list
    xp     = gather(x, plan)                       [R, H], R = assignments to local experts
    gu     = grouped_gemm(xp, w_gate_up)           [R, 2I]  (gate rows then up rows per expert)
    a      = act(gu + b_gate_up)                   [R, I]   SiLU or GPT-OSS clamped SwiGLU
    y      = grouped_gemm(a, w_down)               [R, H]
    out    = combine(y + b_down, w, plan)          [T, H]   weighted sum over the k choices

Assignments to experts of other ranks contribute nothing here; with expert parallelism the
partial outputs are summed across ranks by the caller.

Reference: vllm_neuron/functional/moe/router.py:19-72 (router orderings),
moe_blockwise.py:27 (blockwise mapping), moe_cte.py:35 / moe_tkg.py:17 (expert MLPs),
topk_reduce.py:28 (combine), and the GPT-OSS SwiGLU in vllm_neuron/model/gpt_oss.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import linear as L
from ._ext import ext

ROUTE_TOPK_SOFTMAX = 0
ROUTE_SOFTMAX_TOPK = 1
ROUTE_SIGMOID_TOPK = 2
ACT_SILU = 0
ACT_GPTOSS = 1
EPI_BF16 = 0


@dataclass
class MoEWorkspace:
    """Preallocated device buffers of one MoE block (sized for ``max_tokens`` tokens)."""

    ids: torch.Tensor
    weights: torch.Tensor
    offsets: torch.Tensor
    sorted_src: torch.Tensor
    row_expert: torch.Tensor
    inv_pos: torch.Tensor
    gtiles: torch.Tensor
    gcount: torch.Tensor
    logits: torch.Tensor
    xp: torch.Tensor
    gu: torch.Tensor
    act: torch.Tensor
    y: torch.Tensor

    @classmethod
    def create(cls, max_tokens: int, k: int, num_experts: int, e_local: int, hidden: int,
               inter: int, device, dtype=torch.bfloat16) -> "MoEWorkspace":
        R = max_tokens * k
        gmax = R // 128 + e_local + 1
        i32 = dict(dtype=torch.int32, device=device)
        return cls(
            ids=torch.zeros(max_tokens, k, **i32),
            weights=torch.zeros(max_tokens, k, dtype=torch.float32, device=device),
            offsets=torch.zeros(e_local + 1, **i32),
            sorted_src=torch.zeros(R, **i32),
            row_expert=torch.zeros(R, **i32),
            inv_pos=torch.zeros(R, **i32),
            gtiles=torch.zeros(gmax, 4, **i32),
            gcount=torch.zeros(1, **i32),
            logits=torch.zeros(max_tokens, num_experts, dtype=dtype, device=device),
            xp=torch.zeros(R, hidden, dtype=dtype, device=device),
            gu=torch.zeros(R, 2 * inter, dtype=dtype, device=device),
            act=torch.zeros(R, inter, dtype=dtype, device=device),
            y=torch.zeros(R, hidden, dtype=dtype, device=device),
        )


# ------------------------------------------------------------------------------ oracles
def route_ref(logits: torch.Tensor, k: int, mode: int, renorm: bool = True,
              bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    s = logits.float()
    if bias is not None:
        s = s + bias.float()
    if mode == ROUTE_TOPK_SOFTMAX:
        v, i = torch.topk(s, k, dim=-1)
        return i.to(torch.int32), torch.softmax(v, dim=-1)
    if mode == ROUTE_SOFTMAX_TOPK:
        s = torch.softmax(s, dim=-1)
    else:
        s = torch.sigmoid(s)
    v, i = torch.topk(s, k, dim=-1)
    if renorm:
        v = v / v.sum(-1, keepdim=True)
    return i.to(torch.int32), v


def experts_ref(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, w_gu: torch.Tensor,
                w_down: torch.Tensor, b_gu: torch.Tensor | None = None,
                b_down: torch.Tensor | None = None, act: int = ACT_SILU, alpha: float = 1.702,
                limit: float = 7.0, e_start: int = 0) -> torch.Tensor:
    """fp32 per-token loop: sum_j w_j * expert_{ids_j}(x) over the local experts."""
    T, H = x.shape
    e_local, I2, _ = w_gu.shape
    I = I2 // 2
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    xf = x.float()
    for e in range(e_local):
        tok, j = torch.where(ids.long() == e + e_start)
        if tok.numel() == 0:
            continue
        h = xf[tok] @ w_gu[e].float().t()
        if b_gu is not None:
            h = h + b_gu[e].float()
        g, u = h[:, :I], h[:, I:]
        if act == ACT_GPTOSS:
            g = g.clamp(max=limit)
            u = u.clamp(-limit, limit)
            a = (u + 1) * g * torch.sigmoid(alpha * g)
        else:
            a = torch.nn.functional.silu(g) * u
        y = a @ w_down[e].float().t()
        if b_down is not None:
            y = y + b_down[e].float()
        out.index_add_(0, tok, y * w[tok, j].float()[:, None])
    return out


# ------------------------------------------------------------------------------ kernels
def route(logits: torch.Tensor, k: int, mode: int, renorm: bool = True,
          bias: torch.Tensor | None = None, ids: torch.Tensor | None = None,
          weights: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    T = logits.shape[0]
    if not logits.is_cuda:
        i, v = route_ref(logits, k, mode, renorm, bias)
        if ids is not None:
            ids[:T].copy_(i)
            weights[:T].copy_(v)
            return ids[:T], weights[:T]
        return i, v
    if ids is None:
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        weights = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ids, weights = ids[:T], weights[:T]
    ext().moe_route(logits, bias, k, mode, renorm, ids, weights)
    return ids, weights


def moe_block(x: torch.Tensor, router_w: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor,
              k: int, mode: int, renorm: bool = True, router_b: torch.Tensor | None = None,
              b_gu: torch.Tensor | None = None, b_down: torch.Tensor | None = None,
              act: int = ACT_SILU, alpha: float = 1.702, limit: float = 7.0, e_start: int = 0,
              ws: MoEWorkspace | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed experts for ``x [T, H]`` (see the module docstring); returns ``out [T, H]`` bf16.

    ``w_gu [e_local, 2I, H]`` holds each expert's gate rows followed by its up rows,
    ``w_down [e_local, H, I]``; biases are bf16 ``[e_local, 2I]`` / ``[e_local, H]`` and the
    router bias fp32 ``[E]``.
    """
    T, H = x.shape
    e_local, I2, _ = w_gu.shape
    I = I2 // 2
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    if not x.is_cuda:
        logits = (x.float() @ router_w.float().t()).to(x.dtype)
        ids, w = route_ref(logits, k, mode, renorm, router_b)
        out.copy_(experts_ref(x, ids, w, w_gu, w_down, b_gu, b_down, act, alpha, limit, e_start).to(out.dtype))
        return out
    if T == 0:
        return out
    E = router_w.shape[0]
    if ws is None:
        ws = MoEWorkspace.create(T, k, E, e_local, H, I, x.device)
    logits = ws.logits[:T]
    if T <= L.SKINNY_MAX:
        L.gemm_skinny_bf16(x, router_w, out=logits)
    else:
        L.gemm_out(x, router_w, out=logits)
    ids, w = route(logits, k, mode, renorm, router_b, ws.ids, ws.weights)
    R = T * k
    ext().moe_align(ids, e_start, e_local, ws.offsets, ws.sorted_src, ws.row_expert,
                    ws.inv_pos[:R], ws.gtiles, ws.gcount)
    xp = ws.xp[:R]
    ext().moe_gather(x, ws.sorted_src, k, ws.offsets, xp)
    gu = ws.gu[:R]
    ext().gemm_grouped(xp, w_gu, gu, ws.gtiles, ws.gcount, EPI_BF16, 256)
    a = ws.act[:R]
    ext().moe_act(gu, b_gu, ws.row_expert, ws.offsets, act, alpha, limit, a)
    y = ws.y[:R]
    ext().gemm_grouped(a, w_down, y, ws.gtiles, ws.gcount, EPI_BF16, 256 if H % 256 == 0 else 128)
    ext().moe_combine(y, ws.inv_pos[:R], w, ids, b_down, e_start, out)
    return out
