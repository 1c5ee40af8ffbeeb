"""Snapshot selection and configuration (``VLLM_B200_SNAPSHOT_*``).

A step is captured when any configured rule matches (with no rule, every step up to the
budget):

* ``VLLM_B200_SNAPSHOT_AT_STEP``  step indices of this runner: ``"all"``, ``"3"``, ``"0,5-7"``;
* ``VLLM_B200_SNAPSHOT_TOKENS``   token positions: a step that computes any of them;
* ``VLLM_B200_SNAPSHOT_REQUESTS`` request ids: a step that schedules any of them.

``VLLM_B200_SNAPSHOT_DIR`` enables capture, ``VLLM_B200_SNAPSHOT_MAX_STEPS`` bounds the number
of files, ``VLLM_B200_SNAPSHOT_RANKS`` (``"0,1"``) limits the capturing ranks (default: all),
``VLLM_B200_SNAPSHOT_FORMAT`` is ``pt`` (torch.save) or ``npy`` (raw arrays).  A malformed
selection raises at start-up rather than on the hot path.  Reference: vllm_neuron/snapshot/
config.py (CaptureSelector: call index, generated token and request rules OR'd together).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

FORMATS = ("pt", "npy")


def parse_index_set(raw: str | None, name: str) -> tuple[bool, set[int] | None]:
    """``"all"`` -> (True, None); ``"1,4-6"`` -> (False, {1, 4, 5, 6}); unset -> (False, None)."""
    if raw is None or raw.strip() == "":
        return False, None
    raw = raw.strip()
    if raw.lower() == "all":
        return True, None
    out: set[int] = set()
    for part in raw.split(","):
        part = part.strip()
        try:
            if "-" in part:
                a, b = part.split("-", 1)
                lo, hi = int(a), int(b)
                if hi < lo or lo < 0:
                    raise ValueError
                out.update(range(lo, hi + 1))
            else:
                v = int(part)
                if v < 0:
                    raise ValueError
                out.add(v)
        except ValueError:
            raise ValueError(f"{name}: cannot parse {raw!r} (expected 'all' or e.g. '0,3-5')") from None
    return False, out


@dataclass
class CaptureSelector:
    all_steps: bool = False
    steps: set[int] | None = None
    tokens: set[int] = field(default_factory=set)
    requests: set[str] = field(default_factory=set)

    @property
    def has_rule(self) -> bool:
        return self.all_steps or self.steps is not None or bool(self.tokens) or bool(self.requests)

    def matches(self, step: int, positions: list[tuple[int, int]], request_ids: list[str]) -> bool:
        """``positions``: per scheduled request the half-open range of positions computed."""
        if not self.has_rule:
            return True
        if self.all_steps or (self.steps is not None and step in self.steps):
            return True
        if self.tokens and any(any(lo <= t < hi for t in self.tokens) for lo, hi in positions):
            return True
        return bool(self.requests) and any(r in self.requests for r in request_ids)


@dataclass
class SnapshotConfig:
    directory: str | None = None
    max_steps: int = 64
    ranks: list[int] | None = None
    fmt: str = "pt"
    selector: CaptureSelector = field(default_factory=CaptureSelector)

    @property
    def active(self) -> bool:
        return bool(self.directory)

    def rank_enabled(self, rank: int) -> bool:
        return self.ranks is None or rank in self.ranks

    @classmethod
    def from_env(cls, env=None) -> "SnapshotConfig":
        env = os.environ if env is None else env
        d = env.get("VLLM_B200_SNAPSHOT_DIR") or None
        mx = env.get("VLLM_B200_SNAPSHOT_MAX_STEPS", "64")
        try:
            max_steps = int(mx)
        except ValueError:
            raise ValueError(f"VLLM_B200_SNAPSHOT_MAX_STEPS: not an integer: {mx!r}") from None
        fmt = (env.get("VLLM_B200_SNAPSHOT_FORMAT") or "pt").lower()
        if fmt not in FORMATS:
            raise ValueError(f"VLLM_B200_SNAPSHOT_FORMAT must be one of {FORMATS}, got {fmt!r}")
        ranks = None
        rr = env.get("VLLM_B200_SNAPSHOT_RANKS")
        if rr:
            try:
                ranks = sorted({int(x) for x in rr.split(",") if x.strip()})
            except ValueError:
                ranks = None  # a malformed rank list falls back to every rank
        all_steps, steps = parse_index_set(env.get("VLLM_B200_SNAPSHOT_AT_STEP"), "VLLM_B200_SNAPSHOT_AT_STEP")
        _, toks = parse_index_set(env.get("VLLM_B200_SNAPSHOT_TOKENS"), "VLLM_B200_SNAPSHOT_TOKENS")
        reqs = {x.strip() for x in (env.get("VLLM_B200_SNAPSHOT_REQUESTS") or "").split(",") if x.strip()}
        sel = CaptureSelector(all_steps, steps, toks or set(), reqs)
        return cls(d, max_steps, ranks, fmt, sel)
