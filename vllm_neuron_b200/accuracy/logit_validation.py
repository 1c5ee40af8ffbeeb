"""Logit validation and tensor capture.

* :func:`compare_logits` — per-prompt metrics between two ``[N, V]`` logit sets: max / mean
  absolute error, relative error, argmax agreement, top-k overlap and KL(ref || test) of the
  softmax distributions.
* :func:`validate_against_hf` — runs the engine's prefill logits (``LLMEngine.prompt_logits``)
  against a HuggingFace model on the same prompts.
* :func:`assert_close_three_way` — the oracle rule of the reference's module tests: the
  candidate may deviate from the fp32 oracle only about as much as a bf16 reference does.
* :func:`capture_hidden` — residual-stream states after chosen layers of a prefill (the
  target models' aux-state capture), for layer-by-layer comparison.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class LogitReport:
    max_abs_err: float
    mean_abs_err: float
    rel_err: float
    argmax_agreement: float
    topk_overlap: float
    kl_div: float

    def passed(self, rel_tol: float = 5e-2, min_argmax: float = 0.9) -> bool:
        return self.rel_err <= rel_tol and self.argmax_agreement >= min_argmax


def compare_logits(ref: torch.Tensor, test: torch.Tensor, k: int = 5) -> LogitReport:
    ref, test = ref.float(), test.float()
    d = (test - ref).abs()
    topr = ref.topk(k, -1).indices
    topt = test.topk(k, -1).indices
    overlap = torch.tensor([len(set(a.tolist()) & set(b.tolist())) / k for a, b in zip(topr, topt)]).mean()
    lp_r = torch.log_softmax(ref, -1)
    lp_t = torch.log_softmax(test, -1)
    kl = (lp_r.exp() * (lp_r - lp_t)).sum(-1).mean()
    return LogitReport(float(d.max()), float(d.mean()), float((test - ref).norm() / ref.norm()),
                       float((ref.argmax(-1) == test.argmax(-1)).float().mean()), float(overlap), float(kl))


@torch.no_grad()
def validate_against_hf(engine, hf_model, prompts: list[list[int]], k: int = 5) -> LogitReport:
    """Engine prefill logits of the last prompt position vs. the HF model's."""
    got = engine.prompt_logits(prompts)
    dev = next(hf_model.parameters()).device
    ref = torch.stack([hf_model(torch.tensor([p], device=dev)).logits[0, -1].float().cpu() for p in prompts])
    return compare_logits(ref, got[:, :ref.shape[1]], k)


def assert_close_three_way(oracle_fp32: torch.Tensor, reference_lowp: torch.Tensor,
                           candidate: torch.Tensor, slack: float = 2.0, atol: float = 1e-5):
    """``|candidate - oracle| <= slack * |reference_lowp - oracle| + atol`` in the max norm:
    the candidate may not be worse than ``slack`` times the low-precision reference."""
    o = oracle_fp32.float()
    ref_err = (reference_lowp.float() - o).abs().max().item()
    cand_err = (candidate.float() - o).abs().max().item()
    if cand_err > slack * ref_err + atol:
        raise AssertionError(f"candidate error {cand_err:.3e} exceeds {slack} x reference error "
                             f"{ref_err:.3e} (+{atol})")


@torch.no_grad()
def capture_hidden(engine, prompts: list[list[int]], layers: list[int]) -> torch.Tensor:
    """Residual-stream states ``[tokens, len(layers), H]`` after ``layers`` for a prefill of
    ``prompts`` (all positions, prompts concatenated)."""
    m = engine.model
    old = (list(m.aux_layers), m.aux_hidden)
    m.enable_aux_hidden(layers)
    try:
        engine.prompt_logits(prompts)
        T = sum(len(p) for p in prompts)
        return m.aux_hidden[:T].float().cpu().view(T, len(layers), m.H).clone()
    finally:
        m.aux_layers, m.aux_hidden = old
