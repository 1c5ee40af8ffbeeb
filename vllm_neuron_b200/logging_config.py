"""Logger set-up of the framework (counterpart of vllm_neuron/logging_config.py:14-69): one
``vllm_neuron_b200`` logger tree with a stream handler, its level taken from
``VLLM_B200_LOG_LEVEL``, rank-prefixed records when running under torchrun."""
from __future__ import annotations

import logging
import os
import sys

from . import envs

_FMT = "%(levelname)s %(asctime)s [%(name)s%(rank)s] %(message)s"
_configured = False


class _RankFilter(logging.Filter):
    def filter(self, record: logging.LogRecord) -> bool:
        r = os.environ.get("RANK")
        record.rank = f" r{r}" if r is not None and os.environ.get("WORLD_SIZE", "1") != "1" else ""
        return True


def configure(level: str | None = None) -> logging.Logger:
    """Idempotent; returns the package's root logger."""
    global _configured
    root = logging.getLogger("vllm_neuron_b200")
    lvl = (level or envs.VLLM_B200_LOG_LEVEL or "INFO").upper()
    root.setLevel(getattr(logging, lvl, logging.INFO))
    if not _configured:
        h = logging.StreamHandler(sys.stderr)
        h.setFormatter(logging.Formatter(_FMT, datefmt="%H:%M:%S"))
        h.addFilter(_RankFilter())
        root.addHandler(h)
        root.propagate = False
        _configured = True
    return root


def get_logger(name: str) -> logging.Logger:
    configure()
    if not name.startswith("vllm_neuron_b200"):
        name = "vllm_neuron_b200." + name
    return logging.getLogger(name)
