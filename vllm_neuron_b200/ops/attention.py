"""Paged GQA attention (csrc/attn/paged_attention.cu) and its fp32 torch oracle.

KV cache per layer: ``k_cache, v_cache`` of shape ``[num_blocks, num_kv_heads, block_size,
head_dim]``.  Batch metadata (built on the host once per step, shared by all layers):

* ``q_start [B+1]`` cumulative query lengths, ``seq_lens [B]`` total KV length per sequence
  (cached tokens + tokens of this step), ``block_tables [B, max_blocks]``;
* ``work [W, 2]`` (sequence, first packed row) for the CTAs;
* ``num_splits``: split-KV factor (decode only).

Reference semantics: ``flash_attention`` / ``segmented_attention`` / ``attention_decode``
(vllm_neuron/functional/attention/attention_cte.py:189, attention_segmented_cte.py:657,
attention_decode.py:1266): causal, sliding window, learned sinks, paged prior KV.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from ._ext import ext

FP8_MAX = 448.0   # largest finite float8_e4m3fn value
PREFILL_ROWS = 64
PREFILL_ROWS_TC = 256  # work items of the tcgen05 prefill kernel: two 128-row Q tiles (csrc/attn/fmha_sm100.cu)
DECODE_ROWS = 16


def prefill_rows(head_dim: int, kv_dtype, block_size: int = 16, group: int = 1, dcp_size: int = 1) -> int:
    """Packed query rows per prefill work item: 256 when the tcgen05 kernel serves the step
    (head_dim 128, bf16 cache, block size dividing its 128-token KV tile, GQA group dividing
    its 128-row Q tile, no DCP), else 64 for the mma.sync kernel.  The work list and the kernel
    must agree."""
    import torch

    from .. import envs

    if (head_dim == 128 and kv_dtype == torch.bfloat16 and dcp_size <= 1 and block_size > 0
            and block_size % 8 == 0 and 128 % block_size == 0 and group > 0 and 128 % group == 0
            and not envs.VLLM_B200_DISABLE_TC_ATTENTION):
        return PREFILL_ROWS_TC
    return PREFILL_ROWS
KV_TILE = 64
DECODE_TILE = 16   # tokens per TMA tile of the decode kernel
DECODE_WARPS = 8   # persistent warps per SM of the decode kernel


@dataclass
class AttnWork:
    """Host-side work decomposition for one batch (independent of the layer)."""

    work: np.ndarray  # [W, 2] int32
    decode: bool
    num_splits: int


def build_work(q_lens: np.ndarray, seq_lens: np.ndarray, group: int, num_kv_heads: int,
               num_sms: int = 148, max_splits: int = 16, head_dim: int = 128,
               prefill_rows: int = PREFILL_ROWS) -> AttnWork:
    """Split the batch into CTA work items.

    Decode mode is used when every sequence has at most ``DECODE_ROWS`` packed rows
    (q_len * group); it then also picks a split-KV factor so the grid covers the SMs.
    """
    q_lens = np.asarray(q_lens, dtype=np.int64)
    rows = q_lens * group
    decode = bool(len(rows) > 0 and rows.max() <= DECODE_ROWS)
    if decode:
        work = np.stack([np.arange(len(rows)), np.zeros(len(rows), dtype=np.int64)], 1)
        units = len(rows) * num_kv_heads
        max_len = int(np.max(seq_lens)) if len(rows) else 1
        # csrc/attn/paged_decode.cu: persistent warps (DECODE_WARPS per SM) claim
        # (sequence, KV head, split) units.  Aim for ~3 units per warp for load balance, but
        # keep at least 4 tiles (64 tokens) per split so the per-unit cost stays amortised.
        warps = num_sms * (DECODE_WARPS // 2 if head_dim == 256 else DECODE_WARPS)
        splits = max(1, min(max_splits, math.ceil(3 * warps / max(1, units)),
                            max(1, max_len // (4 * DECODE_TILE))))
        return AttnWork(work.astype(np.int32), True, splits)
    seqs, starts = [], []
    for b, r in enumerate(rows):
        n = int(math.ceil(r / prefill_rows))
        # Longest-first ordering is applied by sorting work items by remaining KV length.
        for t in range(n):
            seqs.append(b)
            starts.append(t * prefill_rows)
    work = np.stack([np.asarray(seqs, dtype=np.int64), np.asarray(starts, dtype=np.int64)], 1) \
        if seqs else np.zeros((0, 2), dtype=np.int64)
    if len(work):
        # Heaviest tiles first: the later rows of the longest sequences see the most KV.
        ctx = np.asarray(seq_lens, dtype=np.int64)[work[:, 0]] - q_lens[work[:, 0]] + work[:, 1] // group
        work = work[np.argsort(-ctx, kind="stable")]
    return AttnWork(work.astype(np.int32), False, 1)


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_tables: torch.Tensor, seq_lens: torch.Tensor, q_start: torch.Tensor,
                    work: torch.Tensor, decode: bool, num_splits: int, scale: float,
                    window: int = 0, sinks: torch.Tensor | None = None,
                    out: torch.Tensor | None = None, part_o: torch.Tensor | None = None,
                    part_lse: torch.Tensor | None = None, k_scale: float = 1.0,
                    v_scale: float = 1.0, splits_dev: torch.Tensor | None = None,
                    prefill_rows: int = PREFILL_ROWS) -> torch.Tensor:
    """Attention of ``q [T, Hq, D]`` over the paged cache; returns ``out [T, Hq, D]``.

    A ``torch.float8_e4m3fn`` cache holds ``K / k_scale`` and ``V / v_scale`` (per-tensor
    scales, the reference's FP8 KV cache: vllm_neuron/utils/dtype_utils.py,
    functional/attention/attention_decode.py:527-651); the kernels dequantize on load.
    ``splits_dev`` (int32 on the device, decode only): the split factor to use, at most
    ``num_splits`` (a CUDA graph captured for the largest context splits each step by its real
    context lengths)."""
    if out is None:
        out = torch.empty_like(q)
    if not q.is_cuda:
        out.copy_(paged_attention_ref(q, k_cache, v_cache, block_tables, seq_lens, q_start,
                                      scale, window, sinks, k_scale, v_scale).to(out.dtype))
        return out
    T, Hq, D = q.shape
    if num_splits > 1 and (part_o is None or part_lse is None):
        part_o = torch.empty((num_splits, T, Hq, D), dtype=torch.float32, device=q.device)
        part_lse = torch.empty((num_splits, T, Hq), dtype=torch.float32, device=q.device)
    ext().paged_attention(q, k_cache, v_cache, block_tables, seq_lens, q_start, work, out,
                          part_o, part_lse, sinks, num_splits, k_cache.shape[1], window, scale,
                          decode, float(k_scale), float(v_scale), splits_dev, None, 1, 0, False,
                          0 if decode else int(prefill_rows))
    return out


def dcp_local_count(n: int, block_size: int, dcp_size: int, dcp_rank: int) -> int:
    """Tokens among global positions ``[0, n)`` held by DCP rank ``dcp_rank``: every window of
    ``dcp_size * block_size`` positions gives each rank one ``block_size`` slice, in rank order
    (the reference's interleave with ``cp_kv_cache_interleave_size == block_size``:
    docs/design/parallelism/dcp.md, "local_filled Computation")."""
    vb = block_size * dcp_size
    full, rem = divmod(int(n), vb)
    return full * block_size + min(max(rem - dcp_rank * block_size, 0), block_size)


def paged_attention_partial(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            block_tables: torch.Tensor, seq_lens: torch.Tensor,
                            q_start: torch.Tensor, work: torch.Tensor, decode: bool,
                            num_splits: int, scale: float, part_o: torch.Tensor,
                            part_lse: torch.Tensor, k_scale: float = 1.0, v_scale: float = 1.0,
                            dcp_seq_lens: torch.Tensor | None = None, dcp_size: int = 1,
                            dcp_rank: int = 0) -> None:
    """Unmerged attention partials ``part_o [S, T, Hq, D]`` (each normalised over its split)
    and ``part_lse [S, T, Hq]`` (log2-sum-exp of the scaled scores, ``-inf`` for an empty
    split); merge them with :func:`attn_combine`.

    Under decode context parallelism ``seq_lens`` are this rank's local token counts and
    ``dcp_seq_lens`` the whole-sequence lengths: each query sees the local keys whose global
    position is at most its own (reference: functional/attention/attention_decode.py:902-1062
    computes the local output and LSE before the cross-rank correction)."""
    if not q.is_cuda:
        o, lse = paged_attention_ref(q, k_cache, v_cache, block_tables, seq_lens, q_start, scale,
                                     k_scale=k_scale, v_scale=v_scale, dcp_seq_lens=dcp_seq_lens,
                                     dcp_size=dcp_size, dcp_rank=dcp_rank, return_lse=True)
        part_o[0].copy_(o)
        part_lse[0].copy_(lse)
        part_lse[1:num_splits].fill_(float("-inf"))
        part_o[1:num_splits].zero_()
        return
    ext().paged_attention(q, k_cache, v_cache, block_tables, seq_lens, q_start, work, q,
                          part_o, part_lse, None, num_splits, k_cache.shape[1], 0, scale,
                          decode, float(k_scale), float(v_scale), None, dcp_seq_lens,
                          int(dcp_size), int(dcp_rank), True, 0)


def attn_combine(part_o: torch.Tensor, part_lse: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge partials ``[S, T, Hq, D]`` / ``[S, T, Hq]`` (log2 domain) into ``out [T, Hq, D]``:
    ``out = sum_s 2^(lse_s - M) O_s / sum_s 2^(lse_s - M)``."""
    S, T, Hq, D = part_o.shape
    if out is None:
        out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=part_o.device)
    if not part_o.is_cuda:
        m = part_lse.amax(0, keepdim=True)
        m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
        w = torch.exp2(part_lse - m)
        den = w.sum(0)
        o = (w[..., None] * part_o).sum(0) / den.clamp_min(1e-30)[..., None]
        out.copy_(o.to(out.dtype))
        return out
    ext().attn_combine(part_o.contiguous(), part_lse.contiguous(), out)
    return out


def paged_attention_ref(q, k_cache, v_cache, block_tables, seq_lens, q_start, scale,
                        window=0, sinks=None, k_scale=1.0, v_scale=1.0, dcp_seq_lens=None,
                        dcp_size=1, dcp_rank=0, return_lse=False):
    """fp32 oracle: gathers each sequence's KV from its blocks and runs masked softmax
    (an fp8 cache is dequantized with its per-tensor scales).  With ``dcp_seq_lens`` the cache
    holds one DCP rank's tokens (``seq_lens`` local counts) and the causal mask is taken in
    global positions; ``return_lse`` also returns the log2-sum-exp of the scaled scores."""
    fp8 = k_cache.dtype == torch.float8_e4m3fn
    ks, vs = (float(k_scale), float(v_scale)) if fp8 else (1.0, 1.0)
    T, Hq, D = q.shape
    Hkv, bs = k_cache.shape[1], k_cache.shape[2]
    G = Hq // Hkv
    out = torch.zeros((T, Hq, D), dtype=torch.float32, device=q.device)
    lse_out = torch.full((T, Hq), float("-inf"), dtype=torch.float32, device=q.device)
    qs = q_start.tolist()
    sl = seq_lens.tolist()
    gl = dcp_seq_lens.tolist() if dcp_seq_lens is not None else sl
    bt = block_tables.cpu()
    for b in range(len(sl)):
        q0, q1, L = qs[b], qs[b + 1], sl[b]
        if q1 == q0:
            continue
        if L == 0:
            continue
        nblk = (L + bs - 1) // bs
        blocks = bt[b, :nblk].to(k_cache.device).long()
        k = k_cache[blocks].float().permute(1, 0, 2, 3).reshape(Hkv, nblk * bs, D)[:, :L] * ks
        v = v_cache[blocks].float().permute(1, 0, 2, 3).reshape(Hkv, nblk * bs, D)[:, :L] * vs
        k = k.repeat_interleave(G, dim=0)
        v = v.repeat_interleave(G, dim=0)
        qq = q[q0:q1].float().permute(1, 0, 2)  # [Hq, n, D]
        s = torch.einsum("hnd,hld->hnl", qq, k) * scale
        n = q1 - q0
        Lg = gl[b]
        pos = torch.arange(Lg - n, Lg, device=q.device)[:, None]
        j = torch.arange(L, device=q.device)
        if dcp_seq_lens is not None:  # global position of each local key
            j = (j // bs) * bs * dcp_size + dcp_rank * bs + j % bs
        j = j[None, :]
        mask = j <= pos
        if window and window > 0:
            mask = mask & (j > pos - window)
        s = s.masked_fill(~mask[None], float("-inf"))
        if sinks is not None:
            sink = sinks.float().view(Hq, 1, 1).expand(Hq, n, 1)
            s = torch.cat([s, sink], dim=-1)
            p = torch.softmax(s, dim=-1)[..., :-1]
        else:
            p = torch.softmax(s, dim=-1)
        p = torch.nan_to_num(p, nan=0.0)  # rows without a visible key (DCP)
        out[q0:q1] = torch.einsum("hnl,hld->hnd", p, v).permute(1, 0, 2)
        if return_lse:
            lse_out[q0:q1] = (torch.logsumexp(s, dim=-1) * (1.0 / math.log(2.0))).permute(1, 0)
    return (out, lse_out) if return_lse else out


def quantize_kv_fp8(x: torch.Tensor, scale: float) -> torch.Tensor:
    """``x / scale`` saturated to the e4m3 range and rounded to ``torch.float8_e4m3fn`` (the
    rule the KV-write kernel applies)."""
    inv = torch.tensor(1.0 / float(scale), dtype=torch.float32)
    return (x.float() * inv).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
