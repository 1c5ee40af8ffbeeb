"""Comparison of captured activations (see :mod:`.tensor_capture`): per request and capture
point, the max / mean absolute error, the relative (Frobenius) error and the cosine similarity
of two runs' rows at the same positions, and the first point along the forward pass where the
two runs part.  Captures are matched by prompt token ids, so the runs may use different request
ids, batchings or parallel layouts.  Reference: vllm_neuron/accuracy/tensor_compare.py (per
module metrics and divergence localisation)."""
from __future__ import annotations

import glob
import os
import re
from dataclasses import dataclass

import torch

from .tensor_capture import prompt_key


@dataclass
class PointReport:
    prompt_index: int
    point: str
    positions: int
    max_abs: float
    mean_abs: float
    rel_err: float
    cosine: float


def compare_tensors(ref: torch.Tensor, test: torch.Tensor) -> dict:
    r, t = ref.float().flatten(1) if ref.dim() > 1 else ref.float()[:, None], \
        test.float().flatten(1) if test.dim() > 1 else test.float()[:, None]
    d = (t - r).abs()
    cos = torch.nn.functional.cosine_similarity(r, t, dim=-1, eps=1e-12).mean()
    return {"max_abs": float(d.max()) if d.numel() else 0.0,
            "mean_abs": float(d.mean()) if d.numel() else 0.0,
            "rel_err": float((t - r).norm() / (r.norm() + 1e-12)),
            "cosine": float(cos) if d.numel() else 1.0}


def _order(point: str) -> tuple:
    """Forward-pass order of capture points: embedding, layers by index, final norm, LM head."""
    if point == "model.embed_tokens":
        return (0, 0)
    m = re.match(r"model\.layers\.(\d+)$", point)
    if m:
        return (1, int(m.group(1)))
    return (2 if point == "model.norm" else 3, 0)


def load_dir(path: str) -> dict[tuple, dict[str, torch.Tensor]]:
    out = {}
    for f in sorted(glob.glob(os.path.join(path, "*.pt"))):
        d = torch.load(f)
        out[prompt_key(d["prompt_token_ids"])] = d["tensors"]
    return out


def compare_captures(ref: dict | str, test: dict | str, points: list[str] | None = None) -> list[PointReport]:
    """Reports for every prompt present in both captures (dicts from :func:`load_dir`, or
    capture directories), in forward-pass order per prompt."""
    ref = load_dir(ref) if isinstance(ref, str) else ref
    test = load_dir(test) if isinstance(test, str) else test
    rows = []
    for i, key in enumerate(k for k in ref if k in test):
        a, b = ref[key], test[key]
        names = sorted((set(a) & set(b)) if points is None else set(points) & set(a) & set(b), key=_order)
        for n in names:
            p = min(a[n].shape[0], b[n].shape[0])
            m = compare_tensors(a[n][:p], b[n][:p])
            rows.append(PointReport(i, n, p, **m))
    return rows


def first_divergence(reports: list[PointReport], rel_tol: float = 2e-2) -> PointReport | None:
    """The earliest point (forward order, any prompt) whose relative error exceeds ``rel_tol``."""
    bad = [r for r in reports if r.rel_err > rel_tol]
    return min(bad, key=lambda r: (_order(r.point), r.prompt_index)) if bad else None


def format_report(reports: list[PointReport]) -> str:
    lines = [f"{'prompt':>6} {'point':<24} {'pos':>5} {'max_abs':>10} {'mean_abs':>10} {'rel_err':>10} {'cosine':>9}"]
    for r in reports:
        lines.append(f"{r.prompt_index:>6} {r.point:<24} {r.positions:>5} {r.max_abs:>10.3e} "
                     f"{r.mean_abs:>10.3e} {r.rel_err:>10.3e} {r.cosine:>9.6f}")
    return "\n".join(lines)
