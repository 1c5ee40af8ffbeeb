"""RMSNorm with fused residual add (csrc/misc/norm_rope.cu) and its torch oracle.

``add_rmsnorm(x, residual, w)``: ``residual += x`` (bf16), ``out = rmsnorm(residual) * w``.
``x`` may be the fp32 accumulation buffer of a split-K / all-reduced projection; it is then
cleared after being read (``clear_x``).  Reference: the fused residual + norm prologues of
the NKI mlp/qkv kernels (vllm_neuron/functional/mlp.py:65, attention/qkv.py:672).
"""
from __future__ import annotations

import torch

from ._ext import ext


def rmsnorm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor | None, w: torch.Tensor, eps: float,
                out: torch.Tensor | None = None, clear_x: bool = False) -> torch.Tensor:
    """In-place ``residual += x``; returns ``rmsnorm(residual)`` (or of ``x`` if no residual)."""
    rows = x.shape[0]
    if out is None:
        out = torch.empty((rows, x.shape[1]), dtype=torch.bfloat16, device=x.device)
    if not x.is_cuda:
        if residual is not None:
            residual.copy_((residual.float() + x.float()).to(residual.dtype))
            src = residual
        else:
            src = x
        out.copy_(rmsnorm_ref(src, w, eps).to(out.dtype))
        if clear_x:
            x.zero_()
        return out
    ext().add_rmsnorm(x, residual, w, out, eps, clear_x and x.dtype == torch.float32)
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    return add_rmsnorm(x, None, w, eps, out=out)
