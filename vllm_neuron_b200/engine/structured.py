"""Structured outputs: per-request grammar matchers (xgrammar) producing a token bitmask that is
applied to the logits before sampling (csrc ``apply_token_bitmask``).

``SamplingParams.structured_outputs`` takes one of ``{"json": schema (dict or str)}``,
``{"json_object": True}``, ``{"regex": pattern}``, ``{"choice": [strings]}`` or
``{"grammar": EBNF}``.  Requests with a grammar run synchronous steps (each bitmask depends on
the previous token) on the eager path; a request whose grammar reaches its end finishes.

Reference: ``enable_structured_outputs`` (vllm_neuron/model/neuron_config.py), the bitmask
attached by the scheduler (vllm_neuron/vllm/core/scheduler.py:940-952) and applied in the
sampler (vllm_neuron/nn/sampler.py:13-169); docs/design/vllm/structured-outputs-and-tool-calling.md.
"""
from __future__ import annotations

import json
import re

import torch


class StructuredOutputManager:
    def __init__(self, vocab_size: int, tokenizer=None, vocab: list[str] | None = None,
                 stop_token_ids: list[int] | None = None):
        import xgrammar as xgr

        self.xgr = xgr
        if tokenizer is not None:
            info = xgr.TokenizerInfo.from_huggingface(tokenizer, vocab_size=vocab_size,
                                                      stop_token_ids=stop_token_ids)
        elif vocab is not None:
            info = xgr.TokenizerInfo(vocab, vocab_type=xgr.VocabType.RAW, vocab_size=vocab_size,
                                     stop_token_ids=stop_token_ids)
        else:
            raise ValueError("structured outputs need a tokenizer (or an explicit vocabulary)")
        self.vocab_size = vocab_size
        self.words = (vocab_size + 31) // 32
        self.compiler = xgr.GrammarCompiler(info)

    def matcher(self, spec: dict):
        c = self.compiler
        if "json" in spec:
            schema = spec["json"]
            g = c.compile_json_schema(schema if isinstance(schema, str) else json.dumps(schema))
        elif spec.get("json_object"):
            g = c.compile_builtin_json_grammar()
        elif "regex" in spec:
            g = c.compile_regex(spec["regex"])
        elif "choice" in spec:
            g = c.compile_regex("(" + "|".join(re.escape(x) for x in spec["choice"]) + ")")
        elif "grammar" in spec:
            g = c.compile_grammar(spec["grammar"])
        else:
            raise ValueError(f"unsupported structured output spec {sorted(spec)}")
        return self.xgr.GrammarMatcher(g)

    def bitmask(self, matchers: list) -> torch.Tensor:
        """int32 ``[len(matchers), words]``; rows without a matcher allow every token."""
        mask = torch.full((len(matchers), self.words), -1, dtype=torch.int32)
        for i, m in enumerate(matchers):
            if m is not None:
                m.fill_next_token_bitmask(mask, i)
        return mask
