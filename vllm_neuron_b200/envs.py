"""Typed environment flags of the framework (prefix ``VLLM_B200_``), read lazily on every
attribute access so that tests and launchers can change them at run time.

The flag set mirrors the reference's ``VLLM_NEURON_*`` flags where the concept carries over to a
GPU (vllm_neuron/envs.py:122-270: log level, debug mode, barrier timeout, KV budget, warm-up
skips, kernel disable switch, runtime input snapshots); Trainium-only flags (CPU compile of NEFFs,
parallel trace, switch collectives, NUMA/EFA) have no counterpart.

    from vllm_neuron_b200 import envs
    if envs.VLLM_B200_DISABLE_CUDA_GRAPHS: ...
"""
from __future__ import annotations

import os
from typing import Any, Callable

PREFIX = "VLLM_B200_"


def _bool(name: str, default: bool) -> Callable[[], bool]:
    def get() -> bool:
        v = os.environ.get(name)
        if v is None or v == "":
            return default
        return v.strip().lower() in ("1", "true", "yes", "on")
    return get


def _int(name: str, default: int | None) -> Callable[[], int | None]:
    def get():
        v = os.environ.get(name)
        return default if v in (None, "") else int(v)
    return get


def _float(name: str, default: float | None) -> Callable[[], float | None]:
    def get():
        v = os.environ.get(name)
        return default if v in (None, "") else float(v)
    return get


def _str(name: str, default: str | None) -> Callable[[], str | None]:
    def get():
        v = os.environ.get(name)
        return default if v in (None, "") else v
    return get


# name -> (getter, description)
_FLAGS: dict[str, tuple[Callable[[], Any], str]] = {}


def _flag(name: str, kind, default, doc: str):
    full = PREFIX + name
    _FLAGS[full] = (kind(full, default), doc)


_flag("LOG_LEVEL", _str, "INFO", "level of the vllm_neuron_b200 loggers (DEBUG/INFO/WARNING/ERROR)")
_flag("DEBUG_MODE", _bool, False,
      "synchronise after every engine step and check the device status word (slow; pinpoints "
      "the failing step)")
_flag("BARRIER_TIMEOUT", _float, 600.0, "seconds a host barrier / process-group collective may wait")
_flag("KV_CACHE_MAX_GIB", _float, None, "cap of the KV-cache budget per GPU (GiB) after profiling")
_flag("MIN_KV_BUDGET_GIB", _float, 0.0, "refuse to start when the KV budget is below this (GiB)")
_flag("SKIP_WARMUP", _bool, False, "skip the warm-up passes at start-up")
_flag("DISABLE_CUDA_GRAPHS", _bool, False, "run decode eagerly (no CUDA-graph capture)")
_flag("DISABLE_PDL", _bool, False,
      "launch kernels in plain stream order instead of programmatic dependent launch "
      "(read by the native library at its first launch)")
_flag("DISABLE_TC_ATTENTION", _bool, False,
      "run prefill attention on the mma.sync kernel instead of the tcgen05 kernel")
_flag("DISABLE_FUSED_COMM", _bool, False,
      "use NCCL collectives instead of the fused peer-memory kernels for TP communication")
_flag("FP4_DECODE_MAX_TOKENS", _int, 64,
      "largest batch that runs MXFP4 experts through the fp4 decode kernel (bf16 grouped GEMM above)")
_flag("PROFILE_DIR", _str, "b200_profile", "output directory of start_profile()/stop_profile()")
_flag("SNAPSHOT_DIR", _str, None, "write the packed inputs of every engine step here (replay/debug)")
_flag("SNAPSHOT_MAX_STEPS", _int, 64, "number of steps captured into SNAPSHOT_DIR")
_flag("HEARTBEAT_TIMEOUT", _float, None,
      "TP > 1: seconds without a peer heartbeat before a step raises PeerFailureError (off if unset)")
_flag("HEARTBEAT_INTERVAL", _float, 0.5, "seconds between heartbeats / peer checks")
_flag("WORKER_TERMINATION_TIMEOUT", _float, 30.0, "seconds shutdown waits for workers")


def __getattr__(name: str):
    if name in _FLAGS:
        return _FLAGS[name][0]()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__():
    return sorted(list(globals()) + list(_FLAGS))


def describe() -> dict[str, tuple[Any, str]]:
    """Current value and description of every flag."""
    return {k: (g(), doc) for k, (g, doc) in _FLAGS.items()}
