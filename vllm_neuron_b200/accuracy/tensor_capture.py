"""Activation capture and replacement for accuracy debugging, keyed by request and position.

The model calls :meth:`CaptureSession.point` at named points of its forward pass:

* ``model.embed_tokens`` -- the residual stream after the embedding,
* ``model.layers.<i>`` -- the residual stream after decoder layer ``i`` (HF ``hidden_states[i+1]``),
* ``model.norm`` -- the final-normed hidden rows,
* ``lm_head`` -- the logits of the rows that sample (one per sampling request).

The runner tells the session which (request, first position, rows) groups make up the batch
before each forward, so every captured row is filed under its request and position: a
capture is independent of how requests were batched, chunked or sharded, and two runs (TP 1 vs
TP 8, fused vs NCCL, this engine vs HF) compare row by row.

* :class:`TensorCapture` keeps ``{request: {point: [positions, features]}}`` on the host and,
  with ``capture_dir``, saves one ``<request>.pt`` per finished request
  (``{"prompt_token_ids", "tensors": {point: fp32 [P, F]}}``).
* :class:`TensorReplacement` overwrites the model's rows at chosen points with golden rows (a
  capture directory of a reference run), matched by the prompt's token ids and the position,
  and the model renormalises the next layer's input from the replaced residual -- so the
  divergence of one layer can be measured with every earlier layer pinned to the reference.

Capture and replacement run the forward eagerly (the engine turns CUDA graphs off).
Reference: vllm_neuron/accuracy/tensor_capture.py (forward hooks, module patterns with
ranges) and tensor_replacement.py (position-indexed golden tensors matched by prompt tokens).
"""
from __future__ import annotations

import glob
import os
import re
from dataclasses import dataclass

import torch


def expand_patterns(patterns: list[str]) -> list[str]:
    """``"model.layers.0-3"`` -> ``model.layers.0 .. model.layers.3`` (a range may sit anywhere
    before a suffix: ``"model.layers.2-4.x"``); other patterns pass through (regexes allowed)."""
    out = []
    rng = re.compile(r"^(.*?)(\d+)-(\d+)(.*)$")
    for p in patterns:
        m = rng.match(p)
        if m and "\\" not in p and "*" not in p:
            pre, a, b, suf = m.groups()
            out.extend(f"{pre}{i}{suf}" for i in range(int(a), int(b) + 1))
        else:
            out.append(p)
    return out


class _Matcher:
    def __init__(self, patterns: list[str] | None):
        pats = expand_patterns(list(patterns or []))
        self.exact = {p for p in pats if re.escape(p) == p}
        self.regex = [re.compile(p) for p in pats if re.escape(p) != p]
        self.all = not pats
        self._cache: dict[str, bool] = {}

    def __call__(self, name: str) -> bool:
        v = self._cache.get(name)
        if v is None:
            v = self.all or name in self.exact or any(r.fullmatch(name) for r in self.regex)
            self._cache[name] = v
        return v


def prompt_key(tokens) -> tuple:
    return tuple(int(t) for t in tokens)


@dataclass
class RowGroup:
    """Rows ``[row, row + n)`` of the batch hold positions ``[pos, pos + n)`` of a request."""

    request_id: str
    prompt: tuple
    pos: int
    n: int
    row: int


class TensorCapture:
    def __init__(self, modules: list[str] | None = None, capture_dir: str | None = None,
                 max_positions: int | None = None):
        self.match = _Matcher(modules)
        self.capture_dir = capture_dir
        self.max_positions = max_positions
        self.store: dict[str, dict[str, dict[int, torch.Tensor]]] = {}
        self.prompts: dict[str, tuple] = {}
        if capture_dir:
            os.makedirs(capture_dir, exist_ok=True)

    def record(self, name: str, t: torch.Tensor, groups: list[RowGroup]):
        if not self.match(name):
            return
        host = t.detach().float().cpu()
        for g in groups:
            d = self.store.setdefault(g.request_id, {}).setdefault(name, {})
            self.prompts[g.request_id] = g.prompt
            for j in range(g.n):
                p = g.pos + j
                if self.max_positions is None or p < self.max_positions:
                    d[p] = host[g.row + j].clone()

    def tensors(self, request_id: str) -> dict[str, torch.Tensor]:
        """``{point: [positions seen, F]}`` in position order (positions must be contiguous
        from 0 for a complete capture)."""
        out = {}
        for name, rows in self.store.get(request_id, {}).items():
            ps = sorted(rows)
            out[name] = torch.stack([rows[p] for p in ps]) if ps else torch.empty(0)
        return out

    def positions(self, request_id: str, name: str) -> list[int]:
        return sorted(self.store.get(request_id, {}).get(name, {}))

    def save(self, request_id: str) -> str | None:
        if not self.capture_dir or request_id not in self.store:
            return None
        path = os.path.join(self.capture_dir, f"{request_id}.pt")
        torch.save({"request_id": request_id, "prompt_token_ids": list(self.prompts.get(request_id, ())),
                    "tensors": self.tensors(request_id)}, path)
        return path

    def drop(self, request_id: str):
        self.store.pop(request_id, None)
        self.prompts.pop(request_id, None)


class TensorReplacement:
    """Golden rows ``{prompt tokens: {point: [P, F]}}`` written over the model's rows."""

    def __init__(self, golden: dict[tuple, dict[str, torch.Tensor]], modules: list[str] | None = None):
        self.golden = {prompt_key(k): v for k, v in golden.items()}
        self.match = _Matcher(modules)
        self.replaced = 0  # rows written (for tests / reports)

    @classmethod
    def from_dir(cls, golden_dir: str, modules: list[str] | None = None) -> "TensorReplacement":
        g = {}
        for f in sorted(glob.glob(os.path.join(golden_dir, "*.pt"))):
            d = torch.load(f)
            g[prompt_key(d["prompt_token_ids"])] = d["tensors"]
        return cls(g, modules)

    def apply(self, name: str, t: torch.Tensor, groups: list[RowGroup]) -> bool:
        if not self.match(name):
            return False
        did = False
        for g in groups:
            src = self.golden.get(g.prompt, {}).get(name)
            if src is None:
                continue
            hi = min(g.pos + g.n, src.shape[0])
            if hi <= g.pos:
                continue
            n = hi - g.pos
            t[g.row:g.row + n].copy_(src[g.pos:hi].to(t.dtype), non_blocking=False)
            self.replaced += n
            did = True
        return did


class CaptureSession:
    """What the model sees: ``point(name, t)`` records and / or replaces; returns True when rows
    of ``t`` were replaced (the caller then recomputes what it derived from ``t``)."""

    def __init__(self, capture: TensorCapture | None = None, replace: TensorReplacement | None = None):
        self.capture = capture
        self.replace = replace
        self.groups: list[RowGroup] = []
        self.logit_groups: list[RowGroup] = []

    def begin(self, groups: list[RowGroup], logit_groups: list[RowGroup]):
        self.groups = groups
        self.logit_groups = logit_groups

    def point(self, name: str, t: torch.Tensor, logits: bool = False) -> bool:
        groups = self.logit_groups if logits else self.groups
        did = False
        if self.replace is not None:
            did = self.replace.apply(name, t, groups)
        if self.capture is not None:
            self.capture.record(name, t, groups)
        return did


def session_from_config(tensor_capture: dict | None, tensor_replacement: dict | None,
                        rank: int = 0) -> CaptureSession | None:
    """``tensor_capture = {"modules": [...], "capture_dir": str, "max_positions": int}`` (only
    rank 0 writes files) and ``tensor_replacement = {"golden_dir": str, "modules": [...]}``."""
    if not tensor_capture and not tensor_replacement:
        return None
    cap = rep = None
    if tensor_capture:
        unknown = set(tensor_capture) - {"modules", "capture_dir", "max_positions"}
        if unknown:
            raise ValueError(f"tensor_capture: unknown keys {sorted(unknown)}")
        cap = TensorCapture(tensor_capture.get("modules"),
                            tensor_capture.get("capture_dir") if rank == 0 else None,
                            tensor_capture.get("max_positions"))
    if tensor_replacement:
        unknown = set(tensor_replacement) - {"golden_dir", "modules"}
        if unknown or "golden_dir" not in tensor_replacement:
            raise ValueError("tensor_replacement needs golden_dir (and optionally modules)")
        rep = TensorReplacement.from_dir(tensor_replacement["golden_dir"], tensor_replacement.get("modules"))
    return CaptureSession(cap, rep)
