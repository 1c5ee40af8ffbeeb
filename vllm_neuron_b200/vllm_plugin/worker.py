"""``B200Worker``: the vLLM V1 worker of the B200 platform (one process per GPU).

vLLM keeps the scheduler, the KV-block manager, stop conditions, detokenisation and the API
server; this worker owns the device: it builds the framework's model for its TP rank, allocates
the paged KV cache with the block count vLLM derives from :meth:`determine_available_memory`,
captures the decode CUDA graphs and runs each step on the sm_100a kernels.  The reference's
counterpart is NeuronWorker (vllm/worker/neuron_worker.py: ``init_device`` :478-525,
``determine_available_memory`` :1043-1063, ``initialize_from_config`` :1083-1101,
``compile_or_warm_up_model`` :1103-1294, ``execute_model``/``sample_tokens`` :1964-2064,
profiler toggle :1993-2059) plus the request bookkeeping of NeuronModelRunner
(``_update_states`` :1915).

Per step vLLM calls ``execute_model(scheduler_output)`` (which only mirrors the request state
and returns ``None``) and then ``sample_tokens(grammar_output)``, which packs the step into the
runner's pinned input buffer, runs it (graph replay for pure decode batches) and returns the
sampled token of every request whose scheduled tokens reach the end of its known sequence.
"""
from __future__ import annotations

import datetime
import time

import numpy as np
import torch
import torch.distributed as dist
from vllm.v1.core.sched.output import SchedulerOutput as VSchedulerOutput
from vllm.v1.kv_cache_interface import FullAttentionSpec, KVCacheSpec
from vllm.v1.outputs import EMPTY_MODEL_RUNNER_OUTPUT, ModelRunnerOutput
from vllm.v1.worker.worker_base import CompilationTimes, WorkerBase

from .. import envs
from ..engine.llm_engine import EngineArgs, build_model, build_runner
from ..engine.request import Request
from ..engine.sampling_params import SamplingParams
from ..engine.scheduler import ScheduledRequest, SchedulerOutput
from ..logging_config import get_logger
from ..parallel import state as ps

log = get_logger("vllm_plugin.worker")

_DTYPES = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}


def convert_sampling_params(sp) -> SamplingParams:
    """vLLM ``SamplingParams`` -> the runner's sampling parameters (stop conditions stay with
    vLLM's scheduler)."""
    if sp is None:
        return SamplingParams(temperature=0.0)
    top_k = getattr(sp, "top_k", 0) or 0
    return SamplingParams(
        temperature=float(sp.temperature), top_k=int(top_k) if top_k > 0 else 0,
        top_p=float(sp.top_p) if sp.top_p is not None else 1.0, min_p=float(getattr(sp, "min_p", 0.0) or 0.0),
        seed=sp.seed, max_tokens=sp.max_tokens, ignore_eos=True, logprobs=getattr(sp, "logprobs", None))


def _async_output_base():
    try:
        from vllm.v1.outputs import AsyncModelRunnerOutput

        return AsyncModelRunnerOutput
    except ImportError:  # pragma: no cover - older vLLM
        return object


class _StepOutput(_async_output_base()):
    """One launched step's ModelRunnerOutput, built when its tokens are back on the host."""

    def __init__(self, handle, req_ids: list[str], samples: list[bool], want_lp: bool):
        self.handle, self.req_ids, self.samples, self.want_lp = handle, req_ids, samples, want_lp

    def get_output(self) -> ModelRunnerOutput:
        toks, lps = self.handle.result()
        n = len(self.req_ids)
        want_lp = self.want_lp
        lp_ids = np.zeros((n, 1), dtype=np.int32) if want_lp else None
        lp_val = np.zeros((n, 1), dtype=np.float32) if want_lp else None
        lp_rank = np.zeros(n, dtype=np.int32) if want_lp else None
        ranks = self.handle.ranks if want_lp else None
        sampled, row = [], 0
        for i, s in enumerate(self.samples):
            if s:
                t = int(toks[row])
                if want_lp:
                    lp_ids[i, 0] = t
                    lp_val[i, 0] = float(lps[row])
                    lp_rank[i] = int(ranks[row])
                row += 1
                sampled.append([t])
            else:
                sampled.append([])
        logprobs = None
        if want_lp:
            from vllm.v1.outputs import LogprobsLists

            logprobs = LogprobsLists(lp_ids, lp_val, lp_rank)
        return ModelRunnerOutput(req_ids=list(self.req_ids),
                                 req_id_to_index={rid: i for i, rid in enumerate(self.req_ids)},
                                 sampled_token_ids=sampled, logprobs=logprobs, prompt_logprobs_dict={},
                                 pooler_output=[])


class B200Worker(WorkerBase):
    def __init__(self, vllm_config, local_rank: int, rank: int, distributed_init_method: str,
                 is_driver_worker: bool = False, **kwargs):
        super().__init__(vllm_config, local_rank, rank, distributed_init_method, is_driver_worker)
        self.reqs: dict[str, Request] = {}
        self._pending: VSchedulerOutput | None = None
        self.model = None
        self.runner = None
        self._profiler = None
        # vLLM's asynchronous scheduling: outputs are returned as AsyncModelRunnerOutput
        self.async_scheduling = bool(getattr(vllm_config.scheduler_config, "async_scheduling", False))

    # ---------------------------------------------------------------- start-up
    def init_device(self) -> None:
        par = self.parallel_config
        world = par.world_size
        if torch.cuda.is_available() and self.device_config.device_type != "cpu":
            self.device = torch.device("cuda", self.local_rank)
            torch.cuda.set_device(self.device)
            backend = "nccl"
        else:
            self.device = torch.device("cpu")
            backend = "gloo"
        if world > 1 and not dist.is_initialized():
            kw = dict(backend=backend, init_method=self.distributed_init_method, world_size=world,
                      rank=self.rank, timeout=datetime.timedelta(seconds=envs.VLLM_B200_BARRIER_TIMEOUT))
            if backend == "nccl":
                kw["device_id"] = self.device
            dist.init_process_group(**kw)
        from ..config import vision_tp_of

        ac = dict(self.vllm_config.additional_config or {})
        opts = ac.get("neuron_config") or ac.get("b200_config") or {}
        ps.initialize_parallel_state(ps.ParallelConfig(world_size=world,
                                                       tensor_parallel_size=par.tensor_parallel_size,
                                                       vision_tp_size=vision_tp_of(ac)))

    def _engine_args(self, load_dummy: bool) -> EngineArgs:
        mc, sc, cc = self.model_config, self.scheduler_config, self.cache_config
        fmt = str(getattr(self.load_config, "load_format", "auto"))
        dummy = load_dummy or fmt.endswith("dummy")
        return EngineArgs(
            model=mc.model, max_num_seqs=sc.max_num_seqs,
            max_num_batched_tokens=sc.max_num_batched_tokens, max_model_len=mc.max_model_len,
            block_size=cc.block_size, load_format="dummy" if dummy else "auto", seed=mc.seed or 0,
            dtype=_DTYPES.get(mc.dtype, "bfloat16"), device=str(self.device),
            additional_config=dict(self.vllm_config.additional_config or {}),
            kv_cache_dtype=str(getattr(cc, "cache_dtype", "auto") or "auto"))

    def load_model(self, *, load_dummy_weights: bool = False) -> None:
        args = self._engine_args(load_dummy_weights)
        tp = ps.get_parallel_state().tp
        t0 = time.perf_counter()
        self.arch, self.model, _, self.device, b200cfg = build_model(args, tp)
        self.runner = build_runner(args, self.model, args.max_model_len, self.device, b200cfg)
        self._free_slots = list(range(self.runner.max_slots - 2, -1, -1))
        log.info("model %s loaded on %s in %.1f s", self.arch.architectures, self.device, time.perf_counter() - t0)

    def get_model(self):
        return self.model

    def get_supported_tasks(self):
        return ("generate",)

    def get_kv_cache_spec(self) -> dict[str, KVCacheSpec]:
        m = self.model
        spec = FullAttentionSpec(block_size=self.cache_config.block_size, num_kv_heads=m.Hkv,
                                 head_size=m.D, dtype=getattr(m, "kv_dtype", m.dtype))
        return {f"layers.{i}.attn": spec for i in range(m.num_kv_layers)}

    def get_cache_block_size_bytes(self) -> int:
        return self.runner.kv_bytes_per_block()

    def determine_available_memory(self) -> int:
        """Bytes for the KV cache: ``gpu_memory_utilization x total`` minus what the weights and
        workspaces hold now, minus a reserve for the decode graphs."""
        if fixed := getattr(self.cache_config, "kv_cache_memory_bytes", None):
            return int(fixed)
        if self.device.type != "cuda":
            return 4096 * self.runner.kv_bytes_per_block()
        torch.cuda.synchronize(self.device)
        free, total = torch.cuda.mem_get_info(self.device)
        budget = total * self.cache_config.gpu_memory_utilization - (total - free) - (2 << 30)
        cap = envs.VLLM_B200_KV_CACHE_MAX_GIB
        if cap is not None:
            budget = min(budget, cap * 2**30)
        return int(max(0, budget))

    def initialize_from_config(self, kv_cache_config) -> None:
        self.runner.allocate_kv_cache(int(kv_cache_config.num_blocks))

    def compile_or_warm_up_model(self) -> CompilationTimes:
        t0 = time.perf_counter()
        if not envs.VLLM_B200_SKIP_WARMUP:
            self.runner.capture_graphs()
        return CompilationTimes(language_model=time.perf_counter() - t0, encoder=0.0)

    # ---------------------------------------------------------------- stepping
    def _update_states(self, so: VSchedulerOutput) -> None:
        for rid in so.finished_req_ids:
            r = self.reqs.pop(rid, None)
            if r is not None and r.slot >= 0:
                self._free_slots.append(r.slot)
        for nr in so.scheduled_new_reqs:
            r = Request(nr.req_id, list(nr.prompt_token_ids or []), convert_sampling_params(nr.sampling_params))
            r.block_ids = list(nr.block_ids[0]) if nr.block_ids else []
            r.num_computed_tokens = nr.num_computed_tokens
            if nr.prompt_embeds is not None:
                r.prompt_embeds = nr.prompt_embeds
            r.slot = self._free_slots.pop()
            self.reqs[nr.req_id] = r
        cd = so.scheduled_cached_reqs
        for i, rid in enumerate(cd.req_ids):
            r = self.reqs[rid]
            nb = cd.new_block_ids[i]
            if rid in cd.resumed_req_ids:
                r.block_ids = list(nb[0]) if nb else []
                toks = cd.all_token_ids.get(rid) if cd.all_token_ids else None
                if toks is not None:
                    # every token is known on the host again (recompute after preemption)
                    r.output_token_ids = list(toks[len(r.prompt_token_ids):])
                    r.num_pending = 0
            elif nb is not None:
                r.block_ids.extend(nb[0])
            r.num_computed_tokens = cd.num_computed_tokens[i]

    def execute_model(self, scheduler_output: VSchedulerOutput):
        self._update_states(scheduler_output)
        if scheduler_output.total_num_scheduled_tokens == 0:
            return EMPTY_MODEL_RUNNER_OUTPUT
        self._pending = scheduler_output
        return None

    def _bitmask(self, out: SchedulerOutput, grammar_output) -> torch.Tensor | None:
        if grammar_output is None or getattr(grammar_output, "grammar_bitmask", None) is None:
            return None
        gm = np.asarray(grammar_output.grammar_bitmask, dtype=np.int32)
        rows = {rid: i for i, rid in enumerate(grammar_output.structured_output_request_ids)}
        S = sum(s.num_logits for s in out.scheduled)
        W = (self.model.V + 31) // 32 if hasattr(self.model, "V") else gm.shape[1]
        full = np.full((S, W), -1, dtype=np.int32)
        w = min(W, gm.shape[1])
        s = 0
        for sr in out.scheduled:
            for _ in range(sr.num_logits):
                j = rows.get(sr.req.request_id)
                if j is not None:
                    full[s, :w] = gm[j, :w]
                s += 1
        return torch.from_numpy(full)

    def sample_tokens(self, grammar_output):
        """Launch the pending step and return its output -- at once (synchronous scheduling) or
        as an ``AsyncModelRunnerOutput`` (vLLM's asynchronous scheduling, which schedules the
        next step before this one's tokens are back).

        All request state moves at launch time: the scheduled tokens count as computed and each
        sampled token counts as pending.  Sampled tokens are never appended on the host: a
        request's next input token is read on the device from its slot (the runner's
        ``-(slot + 1)`` ids), so steps can be launched back to back.  The output object only
        reads this step's host buffer, so vLLM may resolve it from another thread."""
        so, self._pending = self._pending, None
        if so is None:
            return EMPTY_MODEL_RUNNER_OUTPUT
        out = SchedulerOutput()
        for rid, n in so.num_scheduled_tokens.items():
            r = self.reqs[rid]
            start = r.num_computed_tokens
            samples = start + n >= r.num_tokens
            out.scheduled.append(ScheduledRequest(r, start, n, samples))
        out.num_tokens = so.total_num_scheduled_tokens
        want_lp = any(sr.samples and sr.req.sampling_params.logprobs is not None for sr in out.scheduled)
        handle = self.runner.launch(out, want_lp, self._bitmask(out, grammar_output), want_ranks=want_lp)
        req_ids, samples = [], []
        for sr in out.scheduled:
            r = sr.req
            req_ids.append(r.request_id)
            samples.append(sr.samples)
            r.num_computed_tokens = sr.start + sr.num_tokens
            if sr.samples:
                r.num_pending += 1
        result = _StepOutput(handle, req_ids, samples, want_lp)
        if self.async_scheduling:
            return result
        return result.get_output()

    def execute_dummy_batch(self) -> None:
        """An idle data-parallel replica's step: a one-token forward on the null block (no KV
        written, nothing sampled) so that collectives spanning the replicas (the expert-parallel
        exchange of wide-EP MoE layers) stay matched (reference: the DP dummy batch,
        vllm/worker/neuron_model_runner.py:7710)."""
        if self.runner is not None:
            self.runner.dummy_forward()

    def take_draft_token_ids(self):
        return None

    # ---------------------------------------------------------------- misc RPCs
    def profile(self, is_start: bool = True, profile_prefix: str | None = None) -> None:
        import os

        if is_start:
            acts = [torch.profiler.ProfilerActivity.CPU]
            if self.device.type == "cuda":
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self._profiler = torch.profiler.profile(activities=acts)
            self._profiler.start()
        elif self._profiler is not None:
            self._profiler.stop()
            d = envs.VLLM_B200_PROFILE_DIR
            os.makedirs(d, exist_ok=True)
            self._profiler.export_chrome_trace(
                os.path.join(d, f"{profile_prefix or 'trace'}_rank{self.rank}_{int(time.time())}.json"))
            self._profiler = None

    def check_health(self) -> None:
        if self.device is not None and self.device.type == "cuda":
            from ..ops._ext import ext

            code = int(ext().read_status())
            if code:
                from ..exceptions import DeviceStatusError

                raise DeviceStatusError(code, "health check")

    def add_lora(self, lora_request) -> bool:
        raise NotImplementedError("LoRA adapters are not supported by the B200 worker")

    def remove_lora(self, lora_id: int) -> bool:
        return False

    def pin_lora(self, lora_id: int) -> bool:
        return False

    def list_loras(self) -> set[int]:
        return set()

    def reset_mm_cache(self) -> None:
        return None

    def reset_encoder_cache(self) -> None:
        return None

    def shutdown(self) -> None:
        if self.runner is not None:
            self.runner.release_graphs()
