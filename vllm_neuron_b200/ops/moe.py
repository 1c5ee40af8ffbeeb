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
ROUTE_SIGMOID_BIAS_TOPK = 3  # rank by sigmoid + correction bias, weigh by the plain sigmoid
ACT_SILU = 0
ACT_GPTOSS = 1
EPI_BF16 = 0
EPI_BF16_T = 1
# decode-size expert batches (at most this many tokens) run the swapped grouped GEMM
SWAP_MAX_TOKENS = 64


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
    shared_gate: torch.Tensor
    shared: torch.Tensor
    shared_gu: torch.Tensor
    shared_act: torch.Tensor
    xp: torch.Tensor
    gu: torch.Tensor
    act: torch.Tensor
    y: torch.Tensor

    @classmethod
    def create(cls, max_tokens: int, k: int, num_experts: int, e_local: int, hidden: int,
               inter: int, device, dtype=torch.bfloat16, shared_inter: int = 0) -> "MoEWorkspace":
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
            logits=torch.zeros(max_tokens, num_experts + 1, dtype=dtype, device=device),
            shared_gate=torch.zeros(max_tokens, dtype=torch.float32, device=device),
            shared=torch.zeros(max_tokens, hidden, dtype=dtype, device=device),
            shared_gu=torch.zeros(max_tokens if shared_inter else 0, 2 * shared_inter, dtype=dtype, device=device),
            shared_act=torch.zeros(max_tokens if shared_inter else 0, shared_inter, dtype=dtype, device=device),
            xp=torch.zeros(R, hidden, dtype=dtype, device=device),
            gu=torch.zeros(R, 2 * inter, dtype=dtype, device=device),
            act=torch.zeros(R, inter, dtype=dtype, device=device),
            y=torch.zeros(R, hidden, dtype=dtype, device=device),
        )


# ------------------------------------------------------------------------------ oracles
def route_ref(logits: torch.Tensor, k: int, mode: int, renorm: bool = True,
              bias: torch.Tensor | None = None, scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    s = logits.float()
    if mode == ROUTE_SIGMOID_BIAS_TOPK:
        p = torch.sigmoid(s)
        key = p + bias.float() if bias is not None else p
        i = torch.topk(key, k, dim=-1).indices
        v = p.gather(1, i)
        if renorm:
            v = v / (v.sum(-1, keepdim=True) + 1e-20)
        return i.to(torch.int32), v * scale
    if bias is not None:
        s = s + bias.float()
    if mode == ROUTE_TOPK_SOFTMAX:
        v, i = torch.topk(s, k, dim=-1)
        return i.to(torch.int32), torch.softmax(v, dim=-1) * scale
    if mode == ROUTE_SOFTMAX_TOPK:
        s = torch.softmax(s, dim=-1)
    else:
        s = torch.sigmoid(s)
    v, i = torch.topk(s, k, dim=-1)
    if renorm:
        v = v / v.sum(-1, keepdim=True)
    return i.to(torch.int32), v * scale


def _dense(w):
    """bf16 tensor view of a weight (block-FP8 / MXFP4 weights: the bf16 operand the kernels use)."""
    return w.dequant_bf16_ref() if isinstance(w, (L.BlockFP8Weight, L.MXFP4Weight, L.MXFP8Weight)) else w


def experts_ref(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, w_gu: torch.Tensor,
                w_down: torch.Tensor, b_gu: torch.Tensor | None = None,
                b_down: torch.Tensor | None = None, act: int = ACT_SILU, alpha: float = 1.702,
                limit: float = 7.0, e_start: int = 0) -> torch.Tensor:
    """fp32 per-token loop: sum_j w_j * expert_{ids_j}(x) over the local experts."""
    w_gu, w_down = _dense(w_gu), _dense(w_down)
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
          weights: torch.Tensor | None = None, num_experts: int | None = None,
          shared_gate: torch.Tensor | None = None, scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k routing of ``logits [T, E]``.  With ``num_experts = E`` and ``logits [T, E + 1]``
    the last column is a shared expert's gate logit and ``shared_gate[t]`` receives its sigmoid.
    The weights are multiplied by ``scale`` (routed scaling factor)."""
    T = logits.shape[0]
    E = num_experts or logits.shape[1]
    if not logits.is_cuda:
        i, v = route_ref(logits[:, :E], k, mode, renorm, bias, scale)
        if shared_gate is not None:
            shared_gate[:T].copy_(torch.sigmoid(logits[:, E].float()))
        if ids is not None:
            ids[:T].copy_(i)
            weights[:T].copy_(v)
            return ids[:T], weights[:T]
        return i, v
    if ids is None:
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        weights = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ids, weights = ids[:T], weights[:T]
    ext().moe_route(logits, bias, E, k, mode, renorm, ids, weights,
                    shared_gate[:T] if shared_gate is not None else None, float(scale))
    return ids, weights


TILE_COLS = 256
ROUTER_FUSED_MAX_TOKENS = 64  # fused router GEMV + top-k below this batch size


def pack_mxfp4(blocks: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Checkpoint MXFP4 ``blocks [E, N, K/32, 16]`` / ``scales [E, N, K/32]`` -> the kernel's
    weight tiles ``[E, ceil(N/256), K/64, 256*32 + 256*2]`` uint8 (csrc/moe/moe_mxfp4.cu):
    per tile the 256 columns' 32 bytes of a 64-k chunk, each 32-byte group reordered so byte
    ``8t + j`` = original byte ``t + 4j`` (the order lane t of an m16n8k16 B fragment
    consumes), followed by the columns' two e8m0 scales."""
    E, N, G, _ = blocks.shape
    assert G % 2 == 0, "K must be a multiple of 64"
    KC = G // 2
    NB = -(-N // TILE_COLS)
    b = blocks.reshape(E, N, KC, 8, 4).transpose(-1, -2).reshape(E, N, KC, 32)  # fragment order
    sc = scales.reshape(E, N, KC, 2)
    pad = NB * TILE_COLS - N
    if pad:
        b = torch.cat([b, torch.zeros(E, pad, KC, 32, dtype=b.dtype, device=b.device)], 1)
        sc = torch.cat([sc, torch.zeros(E, pad, KC, 2, dtype=sc.dtype, device=sc.device)], 1)
    b = b.view(E, NB, TILE_COLS, KC, 32).permute(0, 1, 3, 2, 4).reshape(E, NB, KC, TILE_COLS * 32)
    sc = sc.view(E, NB, TILE_COLS, KC, 2).permute(0, 1, 3, 2, 4).reshape(E, NB, KC, TILE_COLS * 2)
    return torch.cat([b, sc], -1).contiguous()


def mxfp4_gemm_ref(x: torch.Tensor, rows_expert: torch.Tensor, w_bf16: torch.Tensor) -> torch.Tensor:
    """fp32 oracle of the grouped MXFP4 matmul: row r uses expert ``rows_expert[r]``."""
    return torch.einsum("rk,rnk->rn", x.float(), w_bf16[rows_expert.long()].float())


def shared_expert_ref(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    w_gu, w_down = _dense(w_gu), _dense(w_down)
    I = w_gu.shape[0] // 2
    h = x.float() @ w_gu.float().t()
    return (torch.nn.functional.silu(h[:, :I]) * h[:, I:]) @ w_down.float().t()


def moe_block(x: torch.Tensor, router_w: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor,
              k: int, mode: int, renorm: bool = True, router_b: torch.Tensor | None = None,
              b_gu: torch.Tensor | None = None, b_down: torch.Tensor | None = None,
              act: int = ACT_SILU, alpha: float = 1.702, limit: float = 7.0, e_start: int = 0,
              ws: MoEWorkspace | None = None, out: torch.Tensor | None = None,
              num_experts: int | None = None, shared_gu: torch.Tensor | None = None,
              shared_down: torch.Tensor | None = None, fp4_gu: torch.Tensor | None = None,
              fp4_down: torch.Tensor | None = None, fp4_max_tokens: int = 64,
              routed_scale: float = 1.0, shared_gated: bool = True) -> torch.Tensor:
    """Routed experts for ``x [T, H]`` (see the module docstring); returns ``out [T, H]`` bf16.

    ``w_gu [e_local, 2I, H]`` holds each expert's gate rows followed by its up rows,
    ``w_down [e_local, H, I]``; biases are bf16 ``[e_local, 2I]`` / ``[e_local, H]`` and the
    router bias fp32 ``[E]``.  With a shared expert (``shared_gu [2Is, H]`` gate rows then up
    rows, ``shared_down [H, Is]``) ``router_w`` has ``E + 1`` rows, the last being the shared
    expert's gate, and ``out += sigmoid(x . gate) * shared_expert(x)``; with
    ``shared_gated=False`` the router has ``E`` rows and ``out += shared_expert(x)``.
    ``routed_scale`` multiplies the routing weights (GLM-4.5's routed scaling factor).
    """
    T, H = x.shape
    e_local, I2, _ = w_gu.shape
    I = I2 // 2
    E = num_experts or router_w.shape[0]
    has_shared = shared_gu is not None
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    if not x.is_cuda:
        logits = (x.float() @ router_w.float().t()).to(x.dtype)
        ids, w = route_ref(logits[:, :E], k, mode, renorm, router_b, routed_scale)
        r = experts_ref(x, ids, w, w_gu, w_down, b_gu, b_down, act, alpha, limit, e_start)
        if has_shared:
            gate = torch.sigmoid(logits[:, E:E + 1].float()) if shared_gated else 1.0
            r = r + gate * shared_expert_ref(x, shared_gu, shared_down)
        out.copy_(r.to(out.dtype))
        return out
    if T == 0:
        return out
    if ws is None:
        ws = MoEWorkspace.create(T, k, E, e_local, H, I, x.device,
                                 shared_inter=shared_gu.shape[0] // 2 if has_shared else 0)
    logits = ws.logits[:T, :router_w.shape[0]]
    gated = has_shared and shared_gated
    if T <= ROUTER_FUSED_MAX_TOKENS and H % 8 == 0:
        # decode: router GEMV + top-k in one kernel (one CTA per token)
        ids, w = ws.ids[:T], ws.weights[:T]
        ext().moe_router_topk(x, router_w, router_b, E, k, mode, renorm, float(routed_scale), logits,
                              ids, w, ws.shared_gate[:T] if gated else None)
    else:
        if T <= L.SKINNY_MAX:
            L.gemm_skinny_bf16(x, router_w, out=logits)
        else:
            L.gemm_out(x, router_w, out=logits)
        ids, w = route(logits, k, mode, renorm, router_b, ws.ids, ws.weights, E,
                       ws.shared_gate if gated else None, routed_scale)
    shared = None
    if has_shared:
        from .activation import silu_mul

        gu_sh = L.gemm_out(x, shared_gu, out=ws.shared_gu[:T])
        a_sh = silu_mul(gu_sh, out=ws.shared_act[:T])
        shared = L.gemm_out(a_sh, shared_down, out=ws.shared[:T])
    return _experts_cuda(x, ids, w, w_gu, w_down, k, b_gu, b_down, act, alpha, limit, e_start, ws,
                         out, shared, ws.shared_gate[:T] if gated else None, fp4_gu, fp4_down,
                         fp4_max_tokens)


def moe_experts(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, w_gu: torch.Tensor,
                w_down: torch.Tensor, b_gu: torch.Tensor | None = None,
                b_down: torch.Tensor | None = None, act: int = ACT_SILU, alpha: float = 1.702,
                limit: float = 7.0, e_start: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """The expert half of :func:`moe_block` for given routing ``ids, w [R, k]`` (ids outside
    ``[e_start, e_start + e_local)`` contribute nothing): ``out[r] = sum_j w[r, j] *
    expert_{ids[r, j]}(x[r])`` in bf16.  Used on the rows an expert-parallel dispatch delivered."""
    R, H = x.shape
    k = ids.shape[1]
    if out is None:
        out = torch.empty(R, H, dtype=x.dtype if not x.is_cuda else torch.bfloat16, device=x.device)
    if not x.is_cuda:
        out.copy_(experts_ref(x, ids, w, w_gu, w_down, b_gu, b_down, act, alpha, limit, e_start).to(out.dtype))
        return out
    if R == 0:
        return out
    e_local, I2, _ = w_gu.shape
    ws = MoEWorkspace.create(R, k, e_start + e_local, e_local, H, I2 // 2, x.device)
    return _experts_cuda(x, ids.to(torch.int32).contiguous(), w.float().contiguous(), w_gu, w_down, k,
                         b_gu, b_down, act, alpha, limit, e_start, ws, out, None, None, None, None, 0)


class _MX8TileBufs:
    """MXFP8 buffers of the expert-sorted rows (values and per-entry scale atoms), per (device,
    K); outgrown ones stay referenced because CUDA graphs may have captured them."""

    cache: dict = {}
    retired: list = []

    @classmethod
    def get(cls, rows: int, K: int, entries: int, device):
        key = (str(device), K)
        cur = cls.cache.get(key)
        if cur is None or cur[0].shape[0] < rows or cur[1].shape[0] < entries:
            if cur is not None:
                cls.retired.append(cur)
            r = max(rows, 128 if cur is None else cur[0].shape[0])
            n = max(entries, 1 if cur is None else cur[1].shape[0])
            cur = cls.cache[key] = (torch.empty(r, K, dtype=torch.float8_e4m3fn, device=device),
                                    torch.zeros(n, K // 128, 512, dtype=torch.uint8, device=device))
        return cur[0][:rows], cur[1]

    @classmethod
    def out(cls, rows: int, N: int, device) -> torch.Tensor:
        """bf16 output rows of a row-padded expert stack (the combine reads the first H columns)."""
        key = ("out", str(device), N)
        cur = cls.cache.get(key)
        if cur is None or cur.shape[0] < rows:
            if cur is not None:
                cls.retired.append(cur)
            cur = cls.cache[key] = torch.empty(max(rows, 128), N, dtype=torch.bfloat16, device=device)
        return cur[:rows]


def _mx8_experts_ok(w_gu, w_down) -> bool:
    return (isinstance(w_gu, L.MXFP8Weight) and isinstance(w_down, L.MXFP8Weight)
            and w_gu.q.shape[1] % 128 == 0 and w_down.q.shape[1] % 128 == 0)


def _experts_cuda(x, ids, w, w_gu, w_down, k, b_gu, b_down, act, alpha, limit, e_start, ws, out,
                  shared, shared_gate, fp4_gu, fp4_down, fp4_max_tokens):
    T, H = x.shape
    e_local, I2, _ = w_gu.shape
    I = I2 // 2
    R = T * k
    ext().moe_align(ids, e_start, e_local, ws.offsets, ws.sorted_src, ws.row_expert,
                    ws.inv_pos[:R], ws.gtiles, ws.gcount)
    xp = ws.xp[:R]
    ext().moe_gather(x, ws.sorted_src, k, ws.offsets, xp)
    if _mx8_experts_ok(w_gu, w_down):
        # MXFP8 experts on the block-scaled tensor cores: the sorted rows are quantized to MXFP8
        # with one scale atom per tile-list entry; decode-size batches swap operands (expert
        # weight rows as the 128-row operand, each expert's <= 64 tokens as the N tile)
        # (stacks may be zero-padded: K to 128s, the down projection's rows to 128-row experts)
        gmax = ws.gtiles.shape[0]
        swap = T <= SWAP_MAX_TOKENS
        bn_t = L.skinny_bn(T) if swap else 0
        gt = ws.gtiles[:min(gmax, R)] if swap else ws.gtiles
        xq, sfx = _MX8TileBufs.get(R, w_gu.q.shape[-1], gmax, x.device)
        ext().quant_mx8_tiles(xp, xq, sfx, ws.gtiles, ws.gcount)
        gu = ws.gu[:R]
        if swap:
            ext().gemm_mx8_grouped(w_gu.q, xq, gu, EPI_BF16_T, bn_t, w_gu.sf, sfx, gt, ws.gcount, 1)
        else:
            ext().gemm_mx8_grouped(xq, w_gu.q, gu, EPI_BF16, 128, sfx, w_gu.sf, gt, ws.gcount, 0)
        a = ws.act[:R, :I]
        ext().moe_act(gu, b_gu, ws.row_expert, ws.offsets, act, alpha, limit, a)
        aq, sfa = _MX8TileBufs.get(R, w_down.q.shape[-1], gmax, x.device)
        ext().quant_mx8_tiles(a, aq, sfa, ws.gtiles, ws.gcount)
        nd = w_down.q.shape[1]
        y = ws.y[:R] if nd == H else _MX8TileBufs.out(R, nd, x.device)
        if swap:
            ext().gemm_mx8_grouped(w_down.q, aq, y, EPI_BF16_T, bn_t, w_down.sf, sfa, gt, ws.gcount, 1)
        else:
            ext().gemm_mx8_grouped(aq, w_down.q, y, EPI_BF16, 128, sfa, w_down.sf, gt, ws.gcount, 0)
        ext().moe_combine(y, ws.inv_pos[:R], w, ids, b_down, e_start, shared, shared_gate, out)
        return out
    gu = ws.gu[:R]
    use_fp4 = fp4_gu is not None and T <= fp4_max_tokens
    # decode-size MXFP4 batches: swapped grouped tcgen05 GEMM (expert weight rows as the 128-row
    # operand, the <= 64 tokens of each expert as an N tile), so the 4-bit stream stays
    # memory-bound; an expert holds at most T rows, so each tile-list entry fits one N tile
    swap_fp4 = not use_fp4 and isinstance(w_gu, L.MXFP4Weight) and T <= SWAP_MAX_TOKENS
    bn_t = L.skinny_bn(T) if swap_fp4 else 0
    # every tile-list entry holds >= 1 row: at most R entries exist (bounds the fp4 grid)
    gt = ws.gtiles[:min(ws.gtiles.shape[0], R)]
    if use_fp4:
        ext().moe_mxfp4_gemm(xp, fp4_gu, gu, gt, ws.gcount)
    elif swap_fp4:
        ext().gemm_w8(w_gu.q, xp, gu, EPI_BF16_T, bn_t, 1, w_gu.scales, 3, gt, ws.gcount)
    elif isinstance(w_gu, L.BlockFP8Weight):
        ext().gemm_w8(xp, w_gu.q, gu, EPI_BF16, 256, 1, w_gu.scales, 2, ws.gtiles, ws.gcount)
    elif isinstance(w_gu, L.MXFP4Weight):
        ext().gemm_w8(xp, w_gu.q, gu, EPI_BF16, 256, 1, w_gu.scales, 4, ws.gtiles, ws.gcount)
    else:
        ext().gemm_grouped(xp, w_gu, gu, ws.gtiles, ws.gcount, EPI_BF16, 256)
    a = ws.act[:R, :I]
    ext().moe_act(gu, b_gu, ws.row_expert, ws.offsets, act, alpha, limit, a)
    y = ws.y[:R]
    bn_down = 256 if H % 256 == 0 else 128
    if use_fp4:
        ext().moe_mxfp4_gemm(a, fp4_down, y, gt, ws.gcount)
    elif swap_fp4 and isinstance(w_down, L.MXFP4Weight):
        ext().gemm_w8(w_down.q, a, y, EPI_BF16_T, bn_t, 1, w_down.scales, 3, gt, ws.gcount)
    elif isinstance(w_down, L.BlockFP8Weight):
        ext().gemm_w8(a, w_down.q, y, EPI_BF16, bn_down, 1, w_down.scales, 2, ws.gtiles, ws.gcount)
    elif isinstance(w_down, L.MXFP4Weight):
        ext().gemm_w8(a, w_down.q, y, EPI_BF16, bn_down, 1, w_down.scales, 4, ws.gtiles, ws.gcount)
    else:
        ext().gemm_grouped(a, w_down, y, ws.gtiles, ws.gcount, EPI_BF16, bn_down)
    ext().moe_combine(y, ws.inv_pos[:R], w, ids, b_down, e_start, shared, shared_gate, out)
    return out
