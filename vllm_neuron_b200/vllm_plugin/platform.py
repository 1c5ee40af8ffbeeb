"""``B200Platform``: the out-of-tree vLLM platform of this framework.

What it decides for vLLM (reference: NeuronPlatform, vllm/platform.py:118-938, in particular
``check_and_update_config`` :309-443, ``update_block_size_for_backend`` :174-179,
``get_attn_backend_cls`` :684-691, ``support_hybrid_kv_cache`` :704-715):

* the worker class (``B200Worker``) and a process-per-GPU executor (``mp``, or ``uni`` for
  one GPU in-process);
* no ``torch.compile`` and no vLLM CUDA graphs: the worker captures its own decode graphs
  around the sm_100a kernels;
* KV block size 16 by default (the paged-attention kernels' tile), one KV-cache group (the
  models' sliding-window layers read a window of the shared block table);
* synchronous scheduling (the worker returns each step's tokens from ``sample_tokens``).
"""
from __future__ import annotations

import contextlib
import os

import torch
from vllm.platforms.interface import DeviceCapability, Platform, PlatformEnum

from ..logging_config import get_logger

log = get_logger("vllm_plugin")

WORKER_CLS = "vllm_neuron_b200.vllm_plugin.worker.B200Worker"
ATTN_BACKEND_CLS = "vllm_neuron_b200.vllm_plugin.attention.B200AttentionBackend"
DEFAULT_BLOCK_SIZE = 16


class B200Platform(Platform):
    _enum = PlatformEnum.OOT
    device_name: str = "cuda"
    device_type: str = "cuda"
    dispatch_key: str = "CUDA"
    ray_device_key: str = "GPU"
    dist_backend: str = "nccl"
    device_control_env_var: str = "CUDA_VISIBLE_DEVICES"
    simple_compile_backend: str = "eager"
    supported_quantization: list[str] = ["fp8", "mxfp4"]

    # ---------------------------------------------------------------- device queries
    @classmethod
    def get_device_capability(cls, device_id: int = 0) -> DeviceCapability | None:
        if not torch.cuda.is_available():
            return DeviceCapability(10, 0)
        major, minor = torch.cuda.get_device_capability(device_id)
        return DeviceCapability(major=major, minor=minor)

    @classmethod
    def get_device_name(cls, device_id: int = 0) -> str:
        return torch.cuda.get_device_name(device_id) if torch.cuda.is_available() else "B200"

    @classmethod
    def get_device_uuid(cls, device_id: int = 0) -> str:
        return str(torch.cuda.get_device_properties(device_id).uuid)

    @classmethod
    def get_device_total_memory(cls, device_id: int = 0) -> int:
        return torch.cuda.get_device_properties(device_id).total_memory

    @classmethod
    def set_device(cls, device: torch.device) -> None:
        # a CPU worker (gloo tests) has no device to select
        if torch.device(device).type == "cuda":
            torch.cuda.set_device(device)

    @classmethod
    def inference_mode(cls):
        return torch.inference_mode(mode=True)

    @classmethod
    def is_pin_memory_available(cls) -> bool:
        return True

    @classmethod
    def get_current_memory_usage(cls, device: torch.types.Device | None = None) -> float:
        torch.cuda.reset_peak_memory_stats(device)
        return torch.cuda.max_memory_allocated(device)

    @classmethod
    def device_id_to_physical_device_id(cls, device_id: int) -> int:
        vis = os.environ.get(cls.device_control_env_var)
        if vis:
            return int(vis.split(",")[device_id])
        return device_id

    @classmethod
    def num_compute_units(cls, device_id: int = 0) -> int:
        return torch.cuda.get_device_properties(device_id).multi_processor_count

    # ---------------------------------------------------------------- capabilities
    @classmethod
    def support_hybrid_kv_cache(cls) -> bool:
        return False

    @classmethod
    def support_static_graph_mode(cls) -> bool:
        return False

    @classmethod
    def use_custom_allreduce(cls) -> bool:
        return False

    @classmethod
    def is_async_output_supported(cls, enforce_eager: bool | None) -> bool:
        return False

    @classmethod
    def supports_fp8(cls) -> bool:
        return True

    @classmethod
    def supports_mx(cls) -> bool:
        return True

    @classmethod
    def get_device_communicator_cls(cls) -> str:
        return "vllm.distributed.device_communicators.base_device_communicator.DeviceCommunicatorBase"

    @classmethod
    def get_attn_backend_cls(cls, selected_backend, attn_selector_config=None, *args, **kwargs) -> str:
        return ATTN_BACKEND_CLS

    @classmethod
    def verify_quantization(cls, quant: str) -> None:
        if quant not in cls.supported_quantization:
            raise ValueError(f"quantization {quant!r} is not served by the B200 platform "
                             f"(supported: {cls.supported_quantization})")

    @classmethod
    def validate_request(cls, processed_inputs, params) -> None:
        """Refuse what the worker cannot serve before the request reaches the scheduler
        (reference: NeuronPlatform.validate_request, vllm/platform.py:446-485): pooling requests
        (the worker generates only), prompt logprobs, and top-k logprob lists beyond the sampled
        token (``logprobs=0`` -- the sampled token's logprob and rank -- is served), and logits
        processors (sampling runs fused on the device)."""
        from vllm import SamplingParams as VSamplingParams

        if not isinstance(params, VSamplingParams):
            raise ValueError("the B200 platform serves generation requests only (no pooling params)")
        if getattr(params, "prompt_logprobs", None) is not None:
            raise ValueError("prompt_logprobs are not supported by the B200 platform")
        if params.logprobs is not None and params.logprobs > 0:
            raise ValueError(f"logprobs={params.logprobs}: the B200 platform returns the sampled "
                             "token's logprob only (logprobs=0)")
        if getattr(params, "logits_processors", None):
            raise ValueError("per-request logits processors are not supported by the B200 platform "
                             "(sampling runs fused on the device)")

    # ---------------------------------------------------------------- configuration
    @classmethod
    def update_block_size_for_backend(cls, vllm_config) -> None:
        cache = vllm_config.cache_config
        if getattr(cache, "block_size", None) in (None, 0) or not getattr(cache, "user_specified_block_size", False):
            cache.block_size = DEFAULT_BLOCK_SIZE

    @classmethod
    def check_and_update_config(cls, vllm_config) -> None:
        par = vllm_config.parallel_config
        if par.worker_cls == "auto":
            par.worker_cls = WORKER_CLS
        if par.pipeline_parallel_size != 1:
            raise ValueError("pipeline parallelism is not supported by the B200 platform")
        # component / attention data parallelism needs replicas that step in lockstep, which the
        # framework's own LLM front end drives; under vLLM's engine each DP replica steps alone
        ac = dict(getattr(vllm_config, "additional_config", None) or {})
        opts = ac.get("neuron_config") or ac.get("b200_config") or {}
        for key in ("attention_dp_size", "mlp_dp_size", "embedding_dp_size", "lm_head_dp_size"):
            if int(opts.get(key, 1) or 1) > 1:
                raise ValueError(f"{key} > 1 is served by vllm_neuron_b200.entrypoints.LLM (lockstep "
                                 "replicas); the vLLM plugin runs independent data-parallel replicas")
        if par.distributed_executor_backend not in ("mp", "uni"):
            par.distributed_executor_backend = "uni" if par.world_size == 1 else "mp"
        # vLLM's asynchronous scheduling is served: the worker launches each step with the
        # previous step's tokens read on the device and returns AsyncModelRunnerOutput
        comp = vllm_config.compilation_config
        with contextlib.suppress(Exception):
            from vllm.config import CompilationMode, CUDAGraphMode

            comp.mode = CompilationMode.NONE
            comp.cudagraph_mode = CUDAGraphMode.NONE
        cache = vllm_config.cache_config
        if getattr(cache, "block_size", None) in (None, 0):
            cache.block_size = DEFAULT_BLOCK_SIZE
        if vllm_config.model_config is not None:
            vllm_config.model_config.enforce_eager = True  # vLLM's own graph capture stays off
