"""Exceptions raised by the framework (the reference's single ``CPUCompilationComplete``,
vllm_neuron/exceptions.py, has no counterpart: nothing is compiled ahead of time here)."""
from __future__ import annotations


class B200Error(RuntimeError):
    """Base class."""


class DeviceStatusError(B200Error):
    """A kernel recorded a non-zero status word (a bounded wait expired or a peer failed)."""

    def __init__(self, code: int, where: str = ""):
        self.code = code
        super().__init__(f"device status {code:#x}{' after ' + where if where else ''}: a kernel "
                         "gave up waiting (peer rank failed or a pipeline stalled)")


class KVCacheBudgetError(B200Error):
    """The KV-cache budget left after the model is below the configured minimum."""


class UnsupportedConfigError(B200Error, ValueError):
    """A configuration the framework does not serve."""
