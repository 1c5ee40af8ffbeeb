"""Serving metrics (Prometheus names under the ``vllm_b200:`` prefix).

Counterparts of the reference's metrics (vllm_neuron/metrics.py:23-69): padding histograms
of the token/sequence buckets, executions (here: CUDA-graph replays and eager steps),
startup / model-load time and size.  Prometheus objects are created lazily and only if
``prometheus_client`` is importable; the in-process counters always work.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field

PREFIX = "vllm_b200:"
_PROM = None
_LOCK = threading.Lock()


def _prom():
    global _PROM
    with _LOCK:
        if _PROM is None:
            try:
                import prometheus_client as pc
            except Exception:  # pragma: no cover
                _PROM = {}
                return _PROM
            buckets = [0, 1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096]
            _PROM = {
                "num_seqs_padding": pc.Histogram(PREFIX + "num_seqs_padding", "padded - real sequences per step", buckets=buckets),
                "num_batched_tokens_padding": pc.Histogram(PREFIX + "num_batched_tokens_padding", "padded - real tokens per step", buckets=buckets),
                "graph_replays": pc.Counter(PREFIX + "cuda_graph_replays", "decode steps served by a CUDA graph replay"),
                "startup_time_seconds": pc.Gauge(PREFIX + "startup_time_seconds", "engine start-up time"),
                "model_load_time_seconds": pc.Gauge(PREFIX + "model_load_time_seconds", "weight load time"),
                "model_load_size_bytes": pc.Gauge(PREFIX + "model_load_size_bytes", "bytes of weights loaded"),
                "compilation_time_seconds": pc.Gauge(PREFIX + "compilation_time_seconds", "CUDA graph capture time"),
            }
        return _PROM


@dataclass
class Metrics:
    steps: int = 0
    padded_tokens: int = 0
    padded_seqs: int = 0
    real_tokens: int = 0
    real_seqs: int = 0
    spec_draft_tokens: int = 0      # draft tokens proposed (speculative decoding)
    spec_accepted_tokens: int = 0   # of which accepted by the target model
    extra: dict = field(default_factory=dict)

    @property
    def spec_acceptance_rate(self) -> float:
        return self.spec_accepted_tokens / self.spec_draft_tokens if self.spec_draft_tokens else 0.0

    def observe_padding(self, tokens: int, padded_tokens: int, seqs: int, padded_seqs: int):
        self.real_tokens += tokens
        self.padded_tokens += padded_tokens
        self.real_seqs += seqs
        self.padded_seqs += padded_seqs
        p = _prom()
        if p:
            p["num_batched_tokens_padding"].observe(padded_tokens - tokens)
            p["num_seqs_padding"].observe(padded_seqs - seqs)

    def set_gauge(self, name: str, value: float):
        self.extra[name] = value
        p = _prom()
        if p and name in p:
            p[name].set(value)
