"""Environment flags, logging and exceptions (CPU)."""
import logging

import pytest

from vllm_neuron_b200 import envs
from vllm_neuron_b200.exceptions import DeviceStatusError, KVCacheBudgetError
from vllm_neuron_b200.logging_config import get_logger


def test_flags_are_lazy_and_typed(monkeypatch):
    monkeypatch.delenv("VLLM_B200_DISABLE_CUDA_GRAPHS", raising=False)
    assert envs.VLLM_B200_DISABLE_CUDA_GRAPHS is False
    monkeypatch.setenv("VLLM_B200_DISABLE_CUDA_GRAPHS", "1")
    assert envs.VLLM_B200_DISABLE_CUDA_GRAPHS is True
    monkeypatch.setenv("VLLM_B200_BARRIER_TIMEOUT", "12.5")
    assert envs.VLLM_B200_BARRIER_TIMEOUT == 12.5
    monkeypatch.setenv("VLLM_B200_FP4_DECODE_MAX_TOKENS", "0")
    assert envs.VLLM_B200_FP4_DECODE_MAX_TOKENS == 0
    with pytest.raises(AttributeError):
        envs.VLLM_B200_NOT_A_FLAG
    d = envs.describe()
    assert "VLLM_B200_LOG_LEVEL" in d and all(isinstance(v[1], str) for v in d.values())


def test_logger_level(monkeypatch):
    monkeypatch.setenv("VLLM_B200_LOG_LEVEL", "DEBUG")
    from vllm_neuron_b200 import logging_config

    logging_config.configure()
    log = get_logger("engine")
    assert log.name == "vllm_neuron_b200.engine"
    assert logging.getLogger("vllm_neuron_b200").level == logging.DEBUG
    logging_config.configure("WARNING")


def test_kv_budget_cap(monkeypatch):
    """The KV budget cap and minimum apply to the profiled block count (CPU runner path
    returns a fixed count, so exercise the error type directly)."""
    err = DeviceStatusError(0x105, "step 3")
    assert "0x105" in str(err) and isinstance(err, RuntimeError)
    assert issubclass(KVCacheBudgetError, RuntimeError)
