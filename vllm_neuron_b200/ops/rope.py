"""Rotary embeddings (default / Llama-3 / YaRN tables), per-head q/k RMSNorm and the paged
KV-cache write, fused in one kernel (csrc/misc/norm_rope.cu).

The cos/sin table is ``[max_positions, rot_dim]`` fp32 with ``cos`` in the first half and
``sin`` in the second.  Reference: RoPE variants in vllm_neuron/model/llama3/model.py:206-289
(Llama-3 scaling) and model/gpt_oss/model_bf16.py:142-232 (YaRN with concentration); the
in-kernel cache write of functional/attention/qkv.py:311.
"""
from __future__ import annotations

import math

import torch

from ._ext import ext


def inv_freq_default(rot_dim: int, theta: float) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim))


def inv_freq_llama3(rot_dim: int, theta: float, factor: float, low_freq_factor: float,
                    high_freq_factor: float, original_max_position: int) -> torch.Tensor:
    inv = inv_freq_default(rot_dim, theta)
    low_wl = original_max_position / low_freq_factor
    high_wl = original_max_position / high_freq_factor
    wl = 2 * math.pi / inv
    out = torch.where(wl > low_wl, inv / factor, inv)
    smooth = (original_max_position / wl - low_freq_factor) / (high_freq_factor - low_freq_factor)
    smoothed = (1 - smooth) * out / factor + smooth * out
    medium = (wl >= high_wl) & (wl <= low_wl)
    return torch.where(medium, smoothed, out)


def inv_freq_yarn(rot_dim: int, theta: float, factor: float, original_max_position: int,
                  beta_fast: float = 32.0, beta_slow: float = 1.0,
                  truncate: bool = True) -> tuple[torch.Tensor, float]:
    """YaRN frequencies (Peng et al., 2023) and the attention ("concentration") factor."""
    def corr_dim(num_rot):
        return (rot_dim * math.log(original_max_position / (num_rot * 2 * math.pi))) / (2 * math.log(theta))

    low, high = corr_dim(beta_fast), corr_dim(beta_slow)
    if truncate:
        low, high = math.floor(low), math.ceil(high)
    low, high = max(low, 0), min(high, rot_dim - 1)
    if low == high:
        high += 0.001
    ramp = ((torch.arange(rot_dim // 2, dtype=torch.float64) - low) / (high - low)).clamp(0, 1)
    extra = 1 - ramp
    base = inv_freq_default(rot_dim, theta)
    inv = (base / factor) * (1 - extra) + base * extra
    mscale = 0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0
    return inv, mscale


def cos_sin_table(max_pos: int, rot_dim: int, theta: float, scaling: dict | None = None,
                  device=None) -> torch.Tensor:
    """Build the ``[max_pos, rot_dim]`` cos|sin table for the given HF ``rope_scaling``."""
    mscale = 1.0
    kind = (scaling or {}).get("rope_type", (scaling or {}).get("type", "default")) if scaling else "default"
    if kind == "llama3":
        inv = inv_freq_llama3(rot_dim, theta, scaling["factor"], scaling.get("low_freq_factor", 1.0),
                              scaling.get("high_freq_factor", 4.0),
                              scaling.get("original_max_position_embeddings", 8192))
    elif kind == "yarn":
        orig = scaling.get("original_max_position_embeddings", 4096)
        factor = scaling.get("factor") or max_pos / orig
        inv, mscale = inv_freq_yarn(rot_dim, theta, factor, orig,
                                    scaling.get("beta_fast") or 32.0, scaling.get("beta_slow") or 1.0,
                                    scaling.get("truncate", True))
        if scaling.get("attention_factor") is not None:
            mscale = scaling["attention_factor"]
        elif scaling.get("mscale") and scaling.get("mscale_all_dim"):
            def _m(sc, m):
                return 1.0 if sc <= 1 else 0.1 * m * math.log(sc) + 1.0
            mscale = _m(factor, scaling["mscale"]) / _m(factor, scaling["mscale_all_dim"])
    else:
        inv = inv_freq_default(rot_dim, theta)
    pos = torch.arange(max_pos, dtype=torch.float64)
    f = pos[:, None] * inv[None, :]
    tab = torch.cat([torch.cos(f) * mscale, torch.sin(f) * mscale], dim=1).float()
    return tab.to(device) if device is not None else tab


def rope_kv_write(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                  num_q_heads: int, num_kv_heads: int, head_dim: int, q_out: torch.Tensor,
                  k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                  slot_mapping: torch.Tensor | None = None, q_norm_w: torch.Tensor | None = None,
                  k_norm_w: torch.Tensor | None = None, eps: float = 1e-6,
                  rot_dim: int | None = None, neox: bool = True,
                  clear_input: bool = False, q_pos_scale: tuple[float, float] | None = None,
                  qkv_bias: torch.Tensor | None = None, positions3: torch.Tensor | None = None,
                  mrope_section: tuple[int, int, int] | None = None, k_scale: float = 1.0,
                  v_scale: float = 1.0) -> torch.Tensor:
    """Rotate q/k of ``qkv [T, (Hq + 2 Hkv) * D]``; write rotated q to ``q_out [T, Hq * D]`` and
    k/v into the paged cache at ``slot_mapping`` (int32, negative = skip).  ``q_pos_scale =
    (beta, period)`` multiplies the rotated q by ``1 + beta * log(1 + floor(pos / period))``
    (the long-context query temperature of Ministral-3 / Llama-4 configs).  ``qkv_bias`` (fp32
    ``[(Hq + 2 Hkv) * D]``) is added to the input rows first.  ``positions3 [T, 3]`` with
    ``mrope_section`` selects the interleaved multimodal RoPE of Qwen3-VL.  A
    ``torch.float8_e4m3fn`` cache receives ``k / k_scale`` and ``v / v_scale`` saturated to
    the e4m3 range."""
    rot_dim = rot_dim or head_dim
    beta, period = q_pos_scale if q_pos_scale else (0.0, 1.0)
    if not qkv.is_cuda:
        src = qkv if qkv_bias is None else (qkv[:, :qkv_bias.numel()].float() + qkv_bias.float())
        rope_kv_write_ref(src, positions, cos_sin, num_q_heads, num_kv_heads, head_dim, q_out,
                          k_cache, v_cache, slot_mapping, q_norm_w, k_norm_w, eps, rot_dim, neox,
                          q_pos_scale, positions3, mrope_section, k_scale, v_scale)
        if clear_input:
            qkv.zero_()
        return q_out
    ext().rope_kv_write(qkv, positions, slot_mapping, cos_sin, q_out, k_cache, v_cache,
                        q_norm_w, k_norm_w, eps, num_q_heads, num_kv_heads, head_dim, rot_dim,
                        neox, clear_input and qkv.dtype == torch.float32, float(beta), float(period),
                        qkv_bias, positions3, int(mrope_section[1]) if mrope_section else 0,
                        int(mrope_section[2]) if mrope_section else 0, float(k_scale),
                        float(v_scale))
    return q_out


def apply_rope_ref(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, neox: bool) -> torch.Tensor:
    """x [T, H, rot]; cos/sin [T, rot/2] (fp32)."""
    half = x.shape[-1] // 2
    c, s = cos[:, None, :], sin[:, None, :]
    if neox:
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    x1, x2 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x1 * c - x2 * s
    out[..., 1::2] = x2 * c + x1 * s
    return out


def mrope_cos_sin(cos_sin: torch.Tensor, positions3: torch.Tensor, section) -> torch.Tensor:
    """Per-token ``[T, rot_dim]`` cos|sin rows of the interleaved multimodal RoPE: frequency j
    takes the height position when ``j % 3 == 1 and j < 3 * section[1]``, the width position
    when ``j % 3 == 2 and j < 3 * section[2]``, the temporal position otherwise."""
    half = cos_sin.shape[1] // 2
    j = torch.arange(half)
    comp = torch.zeros(half, dtype=torch.long)
    comp[(j % 3 == 1) & (j < 3 * section[1])] = 1
    comp[(j % 3 == 2) & (j < 3 * section[2])] = 2
    pos = positions3.long()[:, comp]                      # [T, half]
    cos = torch.gather(cos_sin[:, :half][pos.flatten()].view(-1, half, half), 2, j.view(1, -1, 1).expand(pos.shape[0], -1, 1))
    sin = torch.gather(cos_sin[:, half:][pos.flatten()].view(-1, half, half), 2, j.view(1, -1, 1).expand(pos.shape[0], -1, 1))
    return torch.cat([cos[..., 0], sin[..., 0]], 1)


def rope_kv_write_ref(qkv, positions, cos_sin, Hq, Hkv, D, q_out, k_cache, v_cache,
                      slot_mapping, q_norm_w, k_norm_w, eps, rot_dim, neox, q_pos_scale=None,
                      positions3=None, mrope_section=None, k_scale=1.0, v_scale=1.0):
    from .attention import quantize_kv_fp8
    from .norm import rmsnorm_ref

    T = qkv.shape[0]
    x = qkv[:, :(Hq + 2 * Hkv) * D].float().reshape(T, Hq + 2 * Hkv, D)
    q, k, v = x[:, :Hq], x[:, Hq:Hq + Hkv], x[:, Hq + Hkv:]
    if q_norm_w is not None:
        q = rmsnorm_ref(q, q_norm_w, eps).to(torch.bfloat16).float()
    if k_norm_w is not None:
        k = rmsnorm_ref(k, k_norm_w, eps).to(torch.bfloat16).float()
    half = rot_dim // 2
    cs = mrope_cos_sin(cos_sin, positions3, mrope_section) if positions3 is not None else cos_sin[positions.long()]
    cos, sin = cs[:, :half], cs[:, half:rot_dim]
    q = torch.cat([apply_rope_ref(q[..., :rot_dim], cos, sin, neox), q[..., rot_dim:]], -1)
    k = torch.cat([apply_rope_ref(k[..., :rot_dim], cos, sin, neox), k[..., rot_dim:]], -1)
    if q_pos_scale and q_pos_scale[0]:
        beta, period = q_pos_scale
        sc = 1 + beta * torch.log1p(torch.floor(positions.double() / period))
        q = q * sc.float()[:, None, None]
    q_out.view(T, Hq, D).copy_(q.to(q_out.dtype))
    if k_cache is not None and slot_mapping is not None:
        bs = k_cache.shape[2]
        for t in range(T):
            s = int(slot_mapping[t])
            if s < 0:
                continue
            if k_cache.dtype == torch.float8_e4m3fn:
                k_cache[s // bs, :, s % bs] = quantize_kv_fp8(k[t], k_scale)
                v_cache[s // bs, :, s % bs] = quantize_kv_fp8(v[t], v_scale)
            else:
                k_cache[s // bs, :, s % bs] = k[t].to(k_cache.dtype)
                v_cache[s // bs, :, s % bs] = v[t].to(v_cache.dtype)
    return q_out
