"""Gated DeltaNet ops (csrc/deltanet/deltanet.cu) and their fp32 torch oracles.

Batch metadata as for attention: ``q_start [B+1]`` and ``seq_lens [B]`` (int32) of this
step, plus ``slots [B]`` (int32), the per-request index into the state caches
``conv_state [slots, C, K-1]`` (bf16) and ``ssm_state [slots, Hv, dk, dv]`` (fp32).  A
sequence whose context before the step is 0 starts from zero state.

The math follows the gated delta rule (Yang et al., "Gated Delta Networks", 2024) as in the
Qwen3.5/3.6 linear-attention layers; the oracle is a plain per-token loop.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, q_start: torch.Tensor, seq_lens: torch.Tensor,
                  slots: torch.Tensor, state: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``x [T, C]`` -> ``out [T, C] = silu(causal depthwise conv)``; updates ``state``."""
    if not x.is_cuda:
        out.copy_(causal_conv1d_ref(x, w, q_start, seq_lens, slots, state).to(out.dtype))
        return out
    ext().causal_conv1d(x, w, q_start, seq_lens, slots, state, out)
    return out


def causal_conv1d_ref(x, w, q_start, seq_lens, slots, state):
    K = w.shape[1]
    out = torch.zeros(x.shape, dtype=torch.float32)
    qs, sl, sv = q_start.tolist(), seq_lens.tolist(), slots.tolist()
    for b in range(len(sl)):
        t0, t1 = qs[b], qs[b + 1]
        n = t1 - t0
        ctx = sl[b] - n
        prev = state[sv[b]].float().t() if ctx > 0 else torch.zeros(K - 1, x.shape[1])
        seq = torch.cat([prev, x[t0:t1].float()], 0)            # [K-1+n, C]
        y = F.conv1d(seq.t()[None], w.float()[:, None, :], groups=x.shape[1])[0].t()  # [n, C]
        out[t0:t1] = F.silu(y)
        state[sv[b]].copy_(seq[-(K - 1):].t().to(state.dtype))
    return out


def gated_delta_rule(qkv: torch.Tensor, z: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                     A_log: torch.Tensor, dt_bias: torch.Tensor, norm_w: torch.Tensor, eps: float,
                     q_start: torch.Tensor, seq_lens: torch.Tensor, slots: torch.Tensor,
                     state: torch.Tensor, out: torch.Tensor, Hk: int, Hv: int,
                     mode: str = "auto") -> torch.Tensor:
    """Gated delta rule + gated RMSNorm; ``qkv [T, 2 Hk dk + Hv dv]``, ``z [T, Hv dv]``,
    ``a, b [T, Hv]`` -> ``out [T, Hv dv]``; updates ``state``.  ``mode``: "recurrent" (token by
    token), "chunked" (WY form over 64-token chunks, tensor-core intra-chunk products) or
    "auto" (chunked for prefill-sized steps of >= 128 tokens and >= 2 tokens per sequence)."""
    if not qkv.is_cuda:
        out.copy_(gated_delta_rule_ref(qkv, z, a, b, A_log, dt_bias, norm_w, eps, q_start, seq_lens,
                                       slots, state, Hk, Hv).to(out.dtype))
        return out
    ext().gated_delta_rule(qkv, z, a, b, A_log, dt_bias, norm_w, eps, q_start, seq_lens, slots,
                           state, out, Hk, Hv, {"auto": 0, "recurrent": 1, "chunked": 2}[mode])
    return out


def pick_mode(T: int, max_q_len: int, mode: str = "auto") -> str:
    """The kernel choice for a step: the chunked form once some sequence fills a 64-token
    chunk (and the step has >= 128 tokens), the token recurrence otherwise; ``max_q_len``
    0 (unknown) leaves the choice to the op."""
    if mode != "auto" or max_q_len <= 0:
        return mode
    return "chunked" if (max_q_len >= 64 and T >= 128) else "recurrent"


def gated_delta_rule_ref(qkv, z, a, b, A_log, dt_bias, norm_w, eps, q_start, seq_lens, slots,
                         state, Hk, Hv):
    dk, dv = state.shape[2], state.shape[3]
    T = qkv.shape[0]
    x = qkv.float()
    q = x[:, :Hk * dk].view(T, Hk, dk)
    k = x[:, Hk * dk:2 * Hk * dk].view(T, Hk, dk)
    v = x[:, 2 * Hk * dk:2 * Hk * dk + Hv * dv].view(T, Hv, dv)
    rep = Hv // Hk
    q = q.repeat_interleave(rep, 1)
    k = k.repeat_interleave(rep, 1)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    g = torch.exp(-A_log.float().exp() * F.softplus(a.float() + dt_bias.float()))   # [T, Hv]
    beta = torch.sigmoid(b.float())
    o = torch.zeros(T, Hv, dv)
    qs, sl, sv = q_start.tolist(), seq_lens.tolist(), slots.tolist()
    for bi in range(len(sl)):
        t0, t1 = qs[bi], qs[bi + 1]
        ctx = sl[bi] - (t1 - t0)
        S = state[sv[bi]].float().clone() if ctx > 0 else torch.zeros(Hv, dk, dv)
        for t in range(t0, t1):
            S = S * g[t][:, None, None]
            kv = torch.einsum("hkv,hk->hv", S, k[t])
            delta = (v[t] - kv) * beta[t][:, None]
            S = S + k[t][:, :, None] * delta[:, None, :]
            o[t] = torch.einsum("hkv,hk->hv", S, q[t])
        state[sv[bi]].copy_(S)
    o = o.to(torch.bfloat16).float() if qkv.dtype == torch.bfloat16 else o
    var = (o * o).mean(-1, keepdim=True)
    nrm = o * torch.rsqrt(var + eps)
    y = norm_w.float() * nrm * F.silu(z.float().view(T, Hv, dv))
    return y.reshape(T, Hv * dv)


def gated_delta_rule_chunked_ref(qkv, a, b, A_log, dt_bias, q_start, seq_lens, slots, state,
                                 Hk, Hv, chunk: int = 64) -> torch.Tensor:
    """Torch restatement of the chunked (WY) kernels, returning the un-normalised ``o [T, Hv,
    dv]`` (fp32) and updating ``state``.  Per chunk of L tokens with entering state S0 and
    cumulative log decay ``lg``:  A = tril(beta_t e^{lg_t - lg_s} k_t.k_s, -1),
    W = (I + A)^-1 diag(beta e^lg) K,  U = (I + A)^-1 diag(beta) V,  Delta = U - W S0,
    o = diag(e^lg) Q S0 + (tril(e^{lg_t - lg_s}) * Q K^T) Delta,
    S_L = e^{lg_L} S0 + K^T diag(e^{lg_L - lg}) Delta."""
    dk, dv = state.shape[2], state.shape[3]
    T = qkv.shape[0]
    x = qkv.float()
    q = x[:, :Hk * dk].view(T, Hk, dk).repeat_interleave(Hv // Hk, 1)
    k = x[:, Hk * dk:2 * Hk * dk].view(T, Hk, dk).repeat_interleave(Hv // Hk, 1)
    v = x[:, 2 * Hk * dk:2 * Hk * dk + Hv * dv].view(T, Hv, dv)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    lg1 = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())            # [T, Hv]
    beta = torch.sigmoid(b.float())
    o = torch.zeros(T, Hv, dv)
    qs, sl, sv = q_start.tolist(), seq_lens.tolist(), slots.tolist()
    for bi in range(len(sl)):
        t0, t1 = qs[bi], qs[bi + 1]
        if t1 == t0:
            continue
        S = state[sv[bi]].float().clone() if sl[bi] - (t1 - t0) > 0 else torch.zeros(Hv, dk, dv)
        for c0 in range(t0, t1, chunk):
            c1 = min(c0 + chunk, t1)
            L = c1 - c0
            Kc, Qc, Vc = k[c0:c1].transpose(0, 1), q[c0:c1].transpose(0, 1), v[c0:c1].transpose(0, 1)
            lg = torch.cumsum(lg1[c0:c1], 0).t()                                   # [Hv, L]
            bt = beta[c0:c1].t()
            dec = torch.exp(lg[:, :, None] - lg[:, None, :]).tril()                # [Hv, L, L]
            A = (bt[:, :, None] * dec * (Kc @ Kc.transpose(1, 2))).tril(-1)
            inv = torch.linalg.inv(torch.eye(L) + A)
            W = inv @ ((bt * lg.exp())[:, :, None] * Kc)
            U = inv @ (bt[:, :, None] * Vc)
            D = U - W @ S
            o[c0:c1] = (lg.exp()[:, :, None] * (Qc @ S) + (dec * (Qc @ Kc.transpose(1, 2))) @ D).transpose(0, 1)
            S = lg[:, -1:].exp()[:, :, None] * S + Kc.transpose(1, 2) @ (torch.exp(lg[:, -1:] - lg)[:, :, None] * D)
        state[sv[bi]].copy_(S)
    return o


def sigmoid_gate_mul(x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """``x *= sigmoid(gate)`` (the output gate of gated attention)."""
    if not x.is_cuda:
        x.copy_((x.float() * torch.sigmoid(gate.float())).to(x.dtype))
        return x
    ext().sigmoid_gate_mul(x, gate)
    return x
