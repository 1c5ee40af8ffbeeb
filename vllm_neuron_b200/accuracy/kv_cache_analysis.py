"""KV-cache analysis: compare the K / V a serving engine wrote for a prompt against a reference.

The engine's paged cache (``[num_blocks, kv_heads, block_size, head_dim]`` per layer, fp8 caches
dequantized with their per-layer scales) is gathered back into contiguous ``[layers, kv_heads,
tokens, head_dim]`` tensors for one request, and compared token by token, layer by layer and
head by head against an expected set -- typically the teacher-forced KV of the Hugging Face model
on the same prompt (post-RoPE keys, as both caches store them).

Metrics per (token, layer, head): cosine similarity, relative L2 (``||a - e|| / ||e||``) and
relative L-inf (``max|a - e| / max|e|``).  With a ``baseline`` (ground truth, e.g. the fp32 HF
model when ``expected`` is a bf16 reference), errors are taken against the baseline for both the
expected and the actual set, and each token gets the Bhattacharyya coefficient between the two
error distributions (1.0: the actual set errs like the expected one; low values localise where
the engine's KV diverges beyond the reference's own rounding).

Reference behaviour: vllm_neuron/accuracy/kv_cache_analysis.py (``compare_kv_caches`` with the
expected / actual / baseline naming of ``logit_validation``, per-head cosine and relative error
metrics, ``_compute_bc``, ``print_kv_report``).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class KVSet:
    """Contiguous K and V of one prompt: ``[layers, kv_heads, tokens, head_dim]`` (fp32)."""

    k: torch.Tensor
    v: torch.Tensor

    @property
    def num_tokens(self) -> int:
        return int(self.k.shape[2])


def _gather_layer(cache: torch.Tensor, blocks: list[int], n: int, scale: float) -> torch.Tensor:
    """``[num_blocks, H, bs, D]`` paged cache -> ``[H, n, D]`` fp32 for the given block ids."""
    idx = torch.as_tensor(blocks, dtype=torch.long, device=cache.device)
    g = cache.index_select(0, idx)  # [nb, H, bs, D]
    nb, H, bs, D = g.shape
    g = g.permute(1, 0, 2, 3).reshape(H, nb * bs, D)[:, :n]
    return g.float() * float(scale)


def gather_kv(model, blocks: list[int], n: int) -> KVSet:
    """Contiguous KV of the first ``n`` tokens stored in ``blocks`` (every attention layer)."""
    ks, vs = [], []
    for i, (kc, vc) in enumerate(model.kv_caches):
        k_s, v_s = model.kv_scale(i) if hasattr(model, "kv_scale") else (1.0, 1.0)
        ks.append(_gather_layer(kc, blocks, n, k_s).cpu())
        vs.append(_gather_layer(vc, blocks, n, v_s).cpu())
    return KVSet(torch.stack(ks), torch.stack(vs))


def extract_request_kv(llm, prompt_token_ids: list[int]) -> KVSet:
    """Prefill ``prompt_token_ids`` through the engine of ``llm`` (the framework's ``LLM``) and
    return the KV it wrote for the prompt tokens.  The request's blocks are read right after it
    finishes, before any other step can reuse them."""
    from ..engine.sampling_params import SamplingParams

    eng = llm.engine if hasattr(llm, "engine") else llm
    rid = eng.add_request(list(prompt_token_ids), SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True))
    done = eng.run_until_done()
    req = next(r for r in done if r.request_id == rid)
    blocks = list(getattr(req, "freed_block_ids", req.block_ids))
    if eng.device.type == "cuda":
        torch.cuda.synchronize(eng.device)
    return gather_kv(eng.model, blocks, len(prompt_token_ids))


@torch.no_grad()
def hf_kv(hf_model, prompt_token_ids: list[int]) -> KVSet:
    """Teacher-forced KV of a Hugging Face causal LM on the prompt (post-RoPE keys)."""
    dev = next(hf_model.parameters()).device
    ids = torch.tensor([list(prompt_token_ids)], device=dev)
    out = hf_model(input_ids=ids, use_cache=True)
    cache = out.past_key_values
    if hasattr(cache, "layers"):
        pairs = [(l.keys, l.values) for l in cache.layers]
    elif hasattr(cache, "key_cache"):
        pairs = list(zip(cache.key_cache, cache.value_cache))
    else:
        pairs = [(k, v) for k, v in cache]
    k = torch.stack([p[0][0].float().cpu() for p in pairs])
    v = torch.stack([p[1][0].float().cpu() for p in pairs])
    return KVSet(k, v)


def bhattacharyya(e1: np.ndarray, e2: np.ndarray, bins: int = 100) -> float:
    """Bhattacharyya coefficient of two samples' histograms on a shared range (1.0 = identical
    distributions, 0.0 = disjoint)."""
    e1 = np.asarray(e1, dtype=np.float64).ravel()
    e2 = np.asarray(e2, dtype=np.float64).ravel()
    lo = min(e1.min(initial=0.0), e2.min(initial=0.0))
    hi = max(e1.max(initial=0.0), e2.max(initial=0.0))
    if hi <= lo:
        return 1.0
    h1, _ = np.histogram(e1, bins=bins, range=(lo, hi))
    h2, _ = np.histogram(e2, bins=bins, range=(lo, hi))
    p, q = h1 / max(1, h1.sum()), h2 / max(1, h2.sum())
    return float(np.sum(np.sqrt(p * q)))


def _metrics(a: torch.Tensor, e: torch.Tensor) -> dict[str, torch.Tensor]:
    """Per (layer, head, token) metrics of ``a`` against ``e`` (both ``[L, H, T, D]``)."""
    d = a - e
    cos = torch.nn.functional.cosine_similarity(a, e, dim=-1, eps=1e-12)
    l2 = d.norm(dim=-1) / e.norm(dim=-1).clamp_min(1e-12)
    linf = d.abs().amax(dim=-1) / e.abs().amax(dim=-1).clamp_min(1e-12)
    return {"cos": cos, "l2": l2, "linf": linf}


@dataclass
class KVComparison:
    """Per (layer, head, token) metrics for K and V (``[L, H, T]`` tensors); with a baseline also
    the expected set's errors against it and the per-token Bhattacharyya coefficients."""

    k: dict[str, torch.Tensor]
    v: dict[str, torch.Tensor]
    base_k: dict[str, torch.Tensor] | None = None
    base_v: dict[str, torch.Tensor] | None = None
    token_bc_k: list[float] = field(default_factory=list)
    token_bc_v: list[float] = field(default_factory=list)

    def summary(self) -> dict:
        s = {"k_cos_min": float(self.k["cos"].min()), "v_cos_min": float(self.v["cos"].min()),
             "k_l2_max": float(self.k["l2"].max()), "v_l2_max": float(self.v["l2"].max()),
             "k_linf_max": float(self.k["linf"].max()), "v_linf_max": float(self.v["linf"].max())}
        if self.token_bc_k:
            s["k_bc_min"] = float(min(self.token_bc_k))
            s["v_bc_min"] = float(min(self.token_bc_v))
        return s

    def worst(self, which: str = "k", metric: str = "l2", top: int = 5) -> list[tuple[int, int, int, float]]:
        """The ``top`` (layer, head, token, value) entries with the largest error (smallest
        cosine for ``metric='cos'``)."""
        t = (self.k if which == "k" else self.v)[metric]
        flat = -t.flatten() if metric == "cos" else t.flatten()
        vals, idx = torch.topk(flat, min(top, flat.numel()))
        L, H, T = t.shape
        out = []
        for v, i in zip(vals.tolist(), idx.tolist()):
            out.append((i // (H * T), (i // T) % H, i % T, -v if metric == "cos" else v))
        return out


def compare_kv_caches(expected: KVSet, actual: KVSet, baseline: KVSet | None = None,
                      bins: int = 100) -> KVComparison:
    """Compare ``actual`` with ``expected`` (or, with ``baseline``, both against the baseline)."""
    if expected.k.shape != actual.k.shape or expected.v.shape != actual.v.shape:
        raise ValueError(f"KV shapes differ: expected {tuple(expected.k.shape)}, actual {tuple(actual.k.shape)}")
    if baseline is None:
        return KVComparison(_metrics(actual.k, expected.k), _metrics(actual.v, expected.v))
    if baseline.k.shape != actual.k.shape:
        raise ValueError("baseline KV shape differs")
    cmp = KVComparison(_metrics(actual.k, baseline.k), _metrics(actual.v, baseline.v),
                       _metrics(expected.k, baseline.k), _metrics(expected.v, baseline.v))
    for t in range(actual.num_tokens):
        ek = (expected.k[:, :, t] - baseline.k[:, :, t]).numpy()
        ak = (actual.k[:, :, t] - baseline.k[:, :, t]).numpy()
        ev = (expected.v[:, :, t] - baseline.v[:, :, t]).numpy()
        av = (actual.v[:, :, t] - baseline.v[:, :, t]).numpy()
        cmp.token_bc_k.append(bhattacharyya(ek, ak, bins))
        cmp.token_bc_v.append(bhattacharyya(ev, av, bins))
    return cmp


def format_kv_report(cmp: KVComparison, top: int = 5) -> str:
    """Text report: summary line, per-layer worst relative L2 of K and V, and the worst entries."""
    s = cmp.summary()
    lines = ["KV cache comparison: " + ", ".join(f"{k}={v:.4g}" for k, v in s.items())]
    L = cmp.k["l2"].shape[0]
    lines.append("layer  k_l2_max  v_l2_max  k_cos_min  v_cos_min")
    for i in range(L):
        lines.append(f"{i:5d}  {float(cmp.k['l2'][i].max()):8.3g}  {float(cmp.v['l2'][i].max()):8.3g}  "
                     f"{float(cmp.k['cos'][i].min()):9.6f}  {float(cmp.v['cos'][i].min()):9.6f}")
    for which in ("k", "v"):
        for (l, h, t, v) in cmp.worst(which, "l2", top):
            lines.append(f"worst {which.upper()}: layer {l} head {h} token {t} rel-L2 {v:.4g}")
    if cmp.token_bc_k:
        worst_t = int(np.argmin(cmp.token_bc_k))
        lines.append(f"lowest K error-distribution agreement (BC) {min(cmp.token_bc_k):.4f} at token {worst_t}")
    return "\n".join(lines)
