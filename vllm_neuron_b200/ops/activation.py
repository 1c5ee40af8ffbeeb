"""SwiGLU activations (csrc/misc/norm_rope.cu ``silu_mul``) and their torch oracles.

``act = 0``: ``silu(gate) * up`` (Llama / Qwen).  ``act = 1``: the GPT-OSS clamped variant
``(clamp(up, -L, L) + 1) * g * sigmoid(alpha * g)`` with ``g = min(gate, L)``
(reference: SwiGLU alpha/limit in vllm_neuron/model/gpt_oss/model_bf16.py and the
``mlp`` activation clamps of functional/mlp.py:65).
"""
from __future__ import annotations

import torch

from ._ext import ext
from .linear import silu_mul_ref


def swiglu_oai_ref(g: torch.Tensor, u: torch.Tensor, limit: float, alpha: float) -> torch.Tensor:
    g = g.float().clamp(max=limit)
    u = u.float().clamp(-limit, limit)
    return (u + 1) * g * torch.sigmoid(alpha * g)


def silu_mul(inp: torch.Tensor, out: torch.Tensor | None = None, blk: int = 0,
             clear_input: bool = False, act: int = 0, limit: float = 7.0,
             alpha: float = 1.702) -> torch.Tensor:
    T, I2 = inp.shape
    I = I2 // 2
    if out is None:
        out = torch.empty((T, I), dtype=torch.bfloat16, device=inp.device)
    if not inp.is_cuda:
        if act == 0:
            out.copy_(silu_mul_ref(inp, blk).to(out.dtype))
        else:
            if blk > 0:
                v = inp.view(T, I // blk, 2, blk)
                g, u = v[:, :, 0].reshape(T, I), v[:, :, 1].reshape(T, I)
            else:
                g, u = inp[:, :I], inp[:, I:]
            out.copy_(swiglu_oai_ref(g, u, limit, alpha).to(out.dtype))
        if clear_input:
            inp.zero_()
        return out
    ext().silu_mul(inp, out, blk, clear_input and inp.dtype == torch.float32, act, limit, alpha)
    return out
