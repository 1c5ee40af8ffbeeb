"""Bucket utilities: the shape classes the runtime pads to.

On the reference's compiler-driven device every bucket is a separately compiled graph
(vllm_neuron/utils/bucket_utils.py: default power-of-two buckets, validation,
``get_bucket_for_count``, ``get_decode_padded_batch_size``).  Here the decode batch-size buckets
choose which CUDA graphs the model runner captures (a step replays the smallest graph that holds
its batch); the token / sequence buckets of prefill steps only feed the padding metrics, since
eager prefill steps run at their exact size.
"""
from __future__ import annotations

import bisect

# decode graphs captured by default (batch sizes; the runner adds its batch cap)
DEFAULT_DECODE_GRAPH_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128)


def pow2_buckets(lo: int, hi: int) -> list[int]:
    """Powers of two from ``lo`` (rounded up to one) up to ``hi``, with ``hi`` itself last."""
    if lo < 1 or hi < lo:
        raise ValueError(f"bad bucket range [{lo}, {hi}]")
    out, b = [], 1
    while b < lo:
        b <<= 1
    while b < hi:
        out.append(b)
        b <<= 1
    out.append(hi)
    return out


def validate_buckets(buckets, name: str, max_value: int | None = None) -> list[int]:
    """Sorted unique positive integers, none above ``max_value``; raises ValueError otherwise."""
    if buckets is None:
        return []
    vals = list(buckets)
    if not all(isinstance(b, int) and not isinstance(b, bool) and b > 0 for b in vals):
        raise ValueError(f"{name} must be positive integers, got {vals!r}")
    if max_value is not None and any(b > max_value for b in vals):
        raise ValueError(f"{name} {vals!r} exceed {max_value}")
    return sorted(set(vals))


def bucket_for(buckets: list[int] | None, n: int) -> int:
    """Smallest bucket holding ``n`` (``n`` itself when none does or no buckets are set)."""
    if not buckets:
        return n
    i = bisect.bisect_left(buckets, n)
    return buckets[i] if i < len(buckets) else n


def decode_graph_buckets(cap: int, user: list[int] | None = None) -> list[int]:
    """Batch sizes to capture decode CUDA graphs for: ``user`` (e.g. ``num_seqs_buckets``) or the
    defaults, those up to ``cap`` (the runner's largest decode batch), and ``cap`` itself so
    every decode batch has a graph."""
    src = validate_buckets(user, "decode graph buckets") if user else list(DEFAULT_DECODE_GRAPH_BUCKETS)
    out = [b for b in src if b <= cap]
    if cap > 0 and cap not in out:
        out.append(cap)
    return sorted(out)
