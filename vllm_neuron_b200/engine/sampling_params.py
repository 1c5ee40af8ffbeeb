"""Sampling parameters (field names follow ``vllm.SamplingParams`` so either can be passed)."""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class SamplingParams:
    n: int = 1
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    min_p: float = 0.0
    seed: int | None = None
    max_tokens: int | None = 16
    min_tokens: int = 0
    ignore_eos: bool = False
    stop_token_ids: list[int] = field(default_factory=list)
    logprobs: int | None = None
    detokenize: bool = True
    # {"json": schema} | {"json_object": True} | {"regex": r} | {"choice": [..]} | {"grammar": ebnf}
    structured_outputs: dict | None = None

    @classmethod
    def coerce(cls, sp) -> "SamplingParams":
        if sp is None:
            return cls()
        if isinstance(sp, cls):
            return sp
        out = cls()
        for name in ("n", "temperature", "top_p", "top_k", "min_p", "seed", "max_tokens",
                     "min_tokens", "ignore_eos", "logprobs", "detokenize", "structured_outputs"):
            if hasattr(sp, name):
                setattr(out, name, getattr(sp, name))
        stop = getattr(sp, "stop_token_ids", None) or []
        out.stop_token_ids = list(stop)
        if out.top_k is None or out.top_k < 0:
            out.top_k = 0
        return out

    @property
    def greedy(self) -> bool:
        return self.temperature is None or self.temperature <= 1e-5
