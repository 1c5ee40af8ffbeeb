"""vLLM platform plugin: ``vllm serve`` / ``vllm.LLM`` on B200 through this framework.

Installing the package (``pip install -e .``) registers the entry point
``vllm.platform_plugins: b200 = vllm_neuron_b200.vllm_plugin:register``.  vLLM then resolves
its platform to :class:`~vllm_neuron_b200.vllm_plugin.platform.B200Platform`, whose worker
(:class:`~vllm_neuron_b200.vllm_plugin.worker.B200Worker`) runs this framework's models, KV
cache, CUDA graphs and sm_100a kernels under vLLM's own scheduler, KV-block manager, API
server and tokenizer/detokenizer.  This mirrors the reference's bootstrap
(vllm_neuron/__init__.py, vllm_neuron/backend.py:17-93, vllm/platform.py:118-938).

Activation: the plugin claims the platform when a CUDA device of compute capability 10.x is
visible (B200), or when ``VLLM_B200_PLUGIN=1`` forces it; ``VLLM_B200_PLUGIN=0`` disables it.
"""
from __future__ import annotations

import os

PLATFORM_CLS = "vllm_neuron_b200.vllm_plugin.platform.B200Platform"


def _has_sm100() -> bool:
    try:
        import torch

        return torch.cuda.is_available() and any(
            torch.cuda.get_device_capability(i)[0] == 10 for i in range(torch.cuda.device_count()))
    except Exception:
        return False


def register() -> str | None:
    """Entry point of the ``vllm.platform_plugins`` group: the platform class path, or None
    when this machine is not a B200 host."""
    flag = os.environ.get("VLLM_B200_PLUGIN", "")
    if flag == "0":
        return None
    if flag == "1" or _has_sm100():
        return PLATFORM_CLS
    return None
