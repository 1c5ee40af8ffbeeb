"""In-process serving engine: scheduler + model runner + request bookkeeping.

Tensor parallelism is SPMD: every rank (one process per GPU) runs the same deterministic
scheduler on the same requests; sampled tokens are identical on all ranks because every rank
samples the full-vocabulary logits with the same seeds, so no per-step broadcast is needed.
"""
from __future__ import annotations

import itertools
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import envs
from ..config import B200Config, ModelArchConfig, VisionConfig, vision_tp_of
from ..exceptions import DeviceStatusError
from ..metrics import Metrics
from ..parallel.comm import SINGLE, GroupComm
from .block_manager import BlockManager
from .request import Request, RequestStatus
from .sampling_params import SamplingParams
from .scheduler import Scheduler


@dataclass
class EngineArgs:
    model: str | dict | None = None
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    max_model_len: int | None = None
    block_size: int = 16
    gpu_memory_utilization: float = 0.9
    num_gpu_blocks: int | None = None
    enable_prefix_caching: bool = False
    enable_chunked_prefill: bool = True
    load_format: str = "auto"      # "auto" | "dummy"
    seed: int = 0
    dtype: str = "bfloat16"
    device: str = "cuda"
    cuda_graphs: bool = True
    async_scheduling: bool | None = None  # default: on for CUDA devices
    additional_config: dict = field(default_factory=dict)
    kv_cache_dtype: str = "auto"   # "auto" (model dtype) | "fp8" / "fp8_e4m3" (per-layer scales)
    # disaggregated prefill / decode: {"kv_role": "kv_producer" | "kv_consumer",
    # "kv_connector": "TorchDistConnector", "kv_peer_rank": r}
    kv_transfer_config: dict | None = None
    # {"method": "ngram" | "eagle3", "num_speculative_tokens": k, "model": draft checkpoint,
    #  "prompt_lookup_min"/"prompt_lookup_max": n-gram sizes}
    speculative_config: dict | None = None
    # decode context parallelism: every sequence's KV is token-sharded over this many
    # consecutive TP ranks (which share replicated KV heads)
    decode_context_parallel_size: int = 1


@dataclass
class CompletionOutput:
    index: int
    token_ids: list[int]
    text: str = ""
    logprobs: list[float] | None = None
    finish_reason: str | None = None


@dataclass
class RequestOutput:
    request_id: str
    prompt_token_ids: list[int]
    outputs: list[CompletionOutput]
    finished: bool
    metrics: dict = field(default_factory=dict)


def build_model(args: EngineArgs, tp: GroupComm = SINGLE):
    """Resolve the architecture of ``args.model`` (HF config dict, ModelArchConfig or a
    checkpoint directory), build the model for this TP rank and load (or random-init) its
    weights.  Returns ``(arch, model, model_path, device, b200_config)``."""
    from ..models import registry
    from ..utils.checkpoints import load_checkpoint_into

    b200_config = B200Config.from_additional_config(args.additional_config)
    model_path = None
    if isinstance(args.model, dict):
        arch = ModelArchConfig.from_hf(args.model)
    elif isinstance(args.model, ModelArchConfig):
        arch = args.model
    else:
        model_path = args.model
        arch = ModelArchConfig.from_path(args.model)
    device = torch.device(args.device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    dtype = {"bfloat16": torch.bfloat16, "float32": torch.float32, "float16": torch.float16}[args.dtype]
    cls = registry.resolve(arch.architectures)
    max_tok = max(args.max_num_batched_tokens, args.max_num_seqs)
    model = cls(arch, tp=tp, device=device, dtype=dtype, max_tokens=max_tok,
                max_seqs=args.max_num_seqs, block_size=args.block_size)
    vision_tp = vision_tp_of(args.additional_config)
    if vision_tp > 1 and hasattr(model, "set_vision_tp"):
        from ..parallel import state as _ps

        vt = _ps.get_parallel_state().vision_tp
        if vt.world != vision_tp:
            raise ValueError("the parallel state has no vision TP group of this size "
                             "(pass the option to the LLM front end)")
        model.set_vision_tp(vt)
    vcfg = VisionConfig.from_additional_config(args.additional_config)
    if vcfg is not None:
        if not hasattr(model, "configure_vision"):
            raise ValueError(f"vision_neuron_config given for {type(model).__name__}, which has no vision encoder")
        vcfg.resolve_tp_dp(tp.world)
        if vcfg.tp_size != model.visual.tp.world:
            raise ValueError(f"vision tp_size {vcfg.tp_size} does not match the vision TP group "
                             f"({model.visual.tp.world} ranks)")
        model.configure_vision(vcfg, cuda_graphs=b200_config.cuda_graphs)
    cdp = {k: getattr(b200_config, k) for k in ("mlp_dp_size", "embedding_dp_size", "lm_head_dp_size",
                                                "attention_dp_size")}
    if any(v > 1 for v in cdp.values()):
        # component / attention data parallelism (the front end made the replicas and the
        # TP x DP group): re-shard the components before the weights load; replicas step in
        # lockstep and run eagerly (their batch sizes differ per step)
        from ..parallel import state as _ps

        st = _ps.get_parallel_state()
        if not st.config.component_dp:
            raise ValueError("component DP sizes must be passed to the LLM front end (no TP x DP group)")
        if not hasattr(model, "set_component_dp"):
            raise NotImplementedError(f"{type(model).__name__} does not support component data parallelism")
        names = {"mlp_dp_size": "mlp", "embedding_dp_size": "embed", "lm_head_dp_size": "lm_head",
                 "attention_dp_size": "attn"}
        model.set_component_dp({names[k]: st.cdp[v] for k, v in cdp.items() if v > 1})
        if cdp["attention_dp_size"] > 1:
            model.set_attention_dp()
        b200_config.cuda_graphs = False
        b200_config.sequence_parallel = False
        b200_config.sampling_dp = False
    ck_info = {}
    if args.load_format == "dummy" or model_path is None:
        model.init_random(seed=args.seed)
    else:
        ck_info = load_checkpoint_into(model, model_path)
    fp8_scales = _static_fp8_scales(model_path) if model_path is not None else None
    if fp8_scales is not None or b200_config.quantization == "fp8_static":
        if not hasattr(model, "quantize_fp8_static"):
            raise ValueError(f"{type(model).__name__} does not support static FP8 linears")
        model.quantize_fp8_static(fp8_scales)
    elif b200_config.quantization == "fp8_block" or (
            model_path is not None and getattr(arch, "weight_block_size", None)
            and device.type == "cuda" and dtype == torch.bfloat16
            and b200_config.quantization not in ("bf16", "none")):
        # block-scaled FP8 (128 x 128): checkpoints with weight_scale_inv served on the GPU, or
        # random-init weights quantized with quantization="fp8_block" (CPU fp32 runs of a
        # block-FP8 checkpoint keep the exact dequantized weights as the oracle)
        if not hasattr(model, "quantize_block_fp8"):
            raise ValueError(f"{type(model).__name__} does not support block-FP8 linears")
        model.quantize_block_fp8()
    if b200_config.quantization == "mxfp8" or (
            ck_info.get("mxfp8") and device.type == "cuda" and dtype == torch.bfloat16
            and b200_config.quantization not in ("bf16", "none")):
        # MXFP8: random-init weights quantized with quantization="mxfp8", or an MXFP8
        # checkpoint (read as its exact bf16 values) served on the block-scaled tensor cores
        if not hasattr(model, "quantize_mxfp8"):
            raise ValueError(f"{type(model).__name__} does not support MXFP8 linears")
        model.quantize_mxfp8()
    if args.kv_cache_dtype not in (None, "auto"):
        if not hasattr(model, "set_kv_cache_dtype"):
            raise ValueError(f"{type(model).__name__} does not support kv_cache_dtype={args.kv_cache_dtype!r}")
        model.set_kv_cache_dtype(args.kv_cache_dtype, _kv_scales_from_checkpoint(model, model_path))
    real_group = tp.world > 1 and tp.group is not None
    # same-box comparison build: dense projections on cuBLAS (and, with fused_comm off, NCCL)
    from ..ops import linear as _lin

    _lin.set_library_gemm(b200_config.use_cublas_baseline)
    _lin.set_fp8_block_activations(b200_config.fp8_block_activations)
    if b200_config.sequence_parallel and hasattr(model, "sequence_parallel"):
        model.sequence_parallel = True
    if (real_group and device.type == "cuda" and b200_config.fused_comm
            and not envs.VLLM_B200_DISABLE_FUSED_COMM):
        from ..parallel import state as ps

        model.enable_fused_comm(ps.get_parallel_state().cpu, fused_sp=b200_config.fused_sp)
    return arch, model, model_path, device, b200_config


def _static_fp8_scales(model_path) -> dict | None:
    """``{(layer, proj): (weight_scale, input_scale)}`` of a static per-tensor FP8 checkpoint
    (a scalar ``*.weight_scale`` and ``*.input_scale`` per projection, no block scales), else
    None.  Such checkpoints run W8A8 on the FP8 GEMM; block-scaled ones are dequantized."""
    import re

    from ..utils.checkpoints import SafetensorsCheckpoint

    try:
        ck = SafetensorsCheckpoint(model_path)
    except (FileNotFoundError, OSError, ValueError):
        return None
    names = ck.names()
    if any(n.endswith("_scale_inv") for n in names):
        return None
    pat = re.compile(r"layers\.(\d+)\.(?:self_attn|mlp)\.(\w+_proj)\.input_scale$")
    out = {}
    for n in names:
        m = pat.search(n)
        if not m:
            continue
        ws = n[:-len("input_scale")] + "weight_scale"
        if ws not in names:
            continue
        a, b = ck.get(ws), ck.get(n)
        if a.numel() != 1 or b.numel() != 1:
            return None  # per-channel / per-token schemes are not the static per-tensor layout
        out[(int(m.group(1)), m.group(2))] = (float(a.float()), float(b.float()))
    return out or None


def _kv_scales_from_checkpoint(model, model_path) -> list[tuple[float, float]] | None:
    """Per-attention-layer ``self_attn.k_scale`` / ``self_attn.v_scale`` of an fp8-KV checkpoint
    (true value = fp8 byte * scale); layers without them use 1.0 (reference:
    vllm_neuron/model/llama3/model.py:2150-2180)."""
    if model_path is None:
        return None
    from ..utils.checkpoints import SafetensorsCheckpoint

    try:
        ck = SafetensorsCheckpoint(model_path)
    except (FileNotFoundError, OSError, ValueError):
        return None
    names = ck.names()
    pre = "model.language_model." if any(n.startswith("model.language_model.") for n in names) else (
        "model." if any(n.startswith("model.") for n in names) else "")
    layers = getattr(model, "attn_layers", None) or list(range(model.num_kv_layers))
    out = []
    for l in layers:
        pair = []
        for nm in ("k_scale", "v_scale"):
            key = f"{pre}layers.{l}.self_attn.{nm}"
            pair.append(float(ck.get(key).float().reshape(-1)[0]) if key in names else 1.0)
        out.append((pair[0], pair[1]))
    return out


def validate_dcp(arch, model, tp: GroupComm, dcp: int):
    """Decode context parallelism needs replicated KV heads shared by each replica set of
    ``dcp`` consecutive TP ranks, and a model whose attention is full causal softmax attention
    (no sliding window, sinks or linear-attention state) (reference: DCP constraints,
    vllm_neuron/vllm/platform.py:600-660)."""
    W, hkv = tp.world, arch.num_kv_heads
    if W % dcp:
        raise ValueError(f"decode_context_parallel_size={dcp} must divide TP={W}")
    if not (W > hkv and (W // hkv) % dcp == 0):
        raise ValueError(f"DCP={dcp} needs TP={W} > num_kv_heads={hkv} with DCP dividing "
                         f"TP / num_kv_heads (the ranks of a replica set share their KV heads)")
    if not getattr(model, "supports_dcp", False):
        raise NotImplementedError(f"{type(model).__name__} does not support decode context "
                                  "parallelism (sliding windows, sinks or linear attention)")


def build_runner(args: EngineArgs, model, max_model_len: int, device, b200_config):
    """The model runner of ``model`` (KV cache not yet allocated).  Its (scheduler) block size
    is the cache block size times the DCP size."""
    from ..worker.model_runner import ModelRunner

    return ModelRunner(model, max_num_seqs=args.max_num_seqs,
                       max_num_batched_tokens=max(args.max_num_batched_tokens, args.max_num_seqs),
                       max_model_len=max_model_len,
                       block_size=args.block_size * max(1, args.decode_context_parallel_size),
                       cuda_graphs=(args.cuda_graphs and b200_config.cuda_graphs
                                    and getattr(model, "supports_cuda_graphs", True)),
                       device=device, seed=args.seed,
                       # the reference's decode batch buckets select the captured decode graphs
                       graph_buckets=b200_config.num_seqs_buckets)


class LLMEngine:
    def __init__(self, args: EngineArgs, tp: GroupComm = SINGLE):
        self.args = args
        self.tp = tp
        self.arch, self.model, self.model_path, self.device, self.b200_config = build_model(args, tp)
        self.max_model_len = args.max_model_len or self.arch.max_position_embeddings
        max_tok = max(args.max_num_batched_tokens, args.max_num_seqs)
        real_group = tp.world > 1 and tp.group is not None
        self.runner = build_runner(args, self.model, self.max_model_len, self.device, self.b200_config)
        self.runner.sampling_dp = bool(self.b200_config.sampling_dp)
        vcfg = getattr(self.model, "vision_pack", None)
        if vcfg is not None and vcfg.encoder_cache_num_blocks:
            self.runner.encoder_cache_size = vcfg.encoder_cache_num_blocks
        # accuracy tooling: activation capture / golden replacement (eager steps only)
        from ..accuracy.tensor_capture import session_from_config

        self.model.capture = session_from_config(self.b200_config.tensor_capture,
                                                 self.b200_config.tensor_replacement, rank=tp.rank)
        if self.model.capture is not None:
            self.runner.use_graphs = False
        dcp = max(1, int(args.decode_context_parallel_size or 1))
        if dcp > 1:
            from ..parallel import state as _ps

            validate_dcp(self.arch, self.model, tp, dcp)
            group = _ps.get_parallel_state().dcp
            if group.world != dcp:
                raise ValueError("the parallel state has no DCP group of this size "
                                 "(pass decode_context_parallel_size to the LLM front end)")
            self.model.dcp = group
            self.runner.set_dcp(dcp, group.rank)
        nb = args.num_gpu_blocks or self.runner.profile_num_blocks(args.gpu_memory_utilization)
        if real_group and self.device.type == "cuda":
            t = torch.tensor([nb], dtype=torch.int64, device=self.device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN, group=tp.group)
            nb = int(t.item())
        self.runner.allocate_kv_cache(nb)
        self.metrics = Metrics()
        # Models with per-request recurrent state (linear attention) cannot reuse cached KV
        # prefixes: the state after the prefix is not stored with the blocks.
        apc = args.enable_prefix_caching and getattr(self.model, "supports_prefix_caching", True)
        self.block_manager = BlockManager(nb, self.runner.block_size, apc)
        self.scheduler = Scheduler(self.block_manager, args.max_num_seqs, max_tok, self.max_model_len,
                                   enable_chunked_prefill=args.enable_chunked_prefill,
                                   num_batched_tokens_buckets=self.b200_config.num_batched_tokens_buckets,
                                   num_seqs_buckets=self.b200_config.num_seqs_buckets,
                                   metrics=self.metrics)
        self.runner.capture_graphs()
        self._ids = itertools.count()
        self.eos_token_id = self.arch.raw.get("eos_token_id")
        if isinstance(self.eos_token_id, list):
            self.eos_token_id = self.eos_token_id[0] if self.eos_token_id else None
        self.num_steps = 0
        self.async_scheduling = (self.device.type == "cuda" if args.async_scheduling is None
                                 else bool(args.async_scheduling))
        self._inflight = None  # (SchedulerOutput, StepHandle) of the launched, unprocessed step
        self._free_slots = list(range(self.runner.max_slots - 2, -1, -1))
        self.kv_connector = None
        from ..kv_transfer import KVTransferConfig, TorchDistKVConnector

        self.kv_transfer = KVTransferConfig.coerce(args.kv_transfer_config)
        if self.kv_transfer is not None:
            if hasattr(self.model, "conv_state") or not hasattr(self.model, "kv_caches"):
                raise NotImplementedError("KV transfer supports attention-only (KV cache) models")
            from ..parallel import state as _ps

            self.kv_connector = TorchDistKVConnector(self.kv_transfer, meta_group=_ps.get_parallel_state().cpu)
        self.tokenizer = None          # set by the LLM front end when it loads one
        self.structured_vocab = None   # token strings, for grammars on token-id-only engines
        self._structured = None
        self._has_structured = False
        self.proposer = None
        if args.speculative_config:
            self.proposer = self._make_proposer(dict(args.speculative_config))
            self.async_scheduling = False  # drafts depend on the previous step's tokens
        self.monitor = None
        self._last_peer_check = 0.0
        if tp.world > 1 and tp.group is not None and envs.VLLM_B200_HEARTBEAT_TIMEOUT:
            from ..parallel.health import PeerMonitor

            store = torch.distributed.distributed_c10d._get_default_store()
            self.monitor = PeerMonitor(store, torch.distributed.get_rank(), torch.distributed.get_world_size(),
                                       interval_s=envs.VLLM_B200_HEARTBEAT_INTERVAL,
                                       timeout_s=envs.VLLM_B200_HEARTBEAT_TIMEOUT)

    # ---------------------------------------------------------------- requests
    def add_request(self, prompt_token_ids: list[int], params: SamplingParams | None = None,
                    request_id: str | None = None, arrival_time: float | None = None,
                    prompt_embeds: torch.Tensor | None = None, mm=None) -> str:
        """Queue a request.  ``prompt_embeds [P, H]`` (optional) replaces the token embeddings
        of the P prompt positions (reference: merge_prompt_embeds,
        vllm_neuron/functional/prompt_embeds.py:7); ``prompt_token_ids`` then only gives P."""
        params = SamplingParams.coerce(params)
        self.validate_request(params)
        rid = request_id if request_id is not None else str(next(self._ids))
        req = Request(rid, list(prompt_token_ids), params, eos_token_id=self.eos_token_id,
                      prompt_embeds=prompt_embeds, mm=mm)
        if params.structured_outputs:
            req.matcher = self.structured_outputs().matcher(params.structured_outputs)
            self._has_structured = True
        if arrival_time is not None:
            req.arrival_time = arrival_time
        if not self._free_slots:
            raise RuntimeError("too many unfinished requests for the device token slots")
        req.slot = self._free_slots.pop()
        try:
            self.scheduler.add_request(req)
        except Exception:
            self._free_slots.append(req.slot)
            raise
        return rid

    def validate_request(self, params: SamplingParams):
        """Refuse what this engine was configured not to serve (reference: the platform's
        request validation, vllm_neuron/vllm/platform.py:446-485): structured outputs when
        ``enable_structured_outputs`` is off, and more logprobs than ``max_logprobs`` (0 = no
        cap; only the sampled token's logprob is returned)."""
        cfg = self.b200_config
        if params.structured_outputs and not cfg.enable_structured_outputs:
            raise ValueError("structured outputs are disabled (enable_structured_outputs=False)")
        if params.logprobs and cfg.max_logprobs and params.logprobs > cfg.max_logprobs:
            raise ValueError(f"logprobs={params.logprobs} exceeds max_logprobs={cfg.max_logprobs}")
        if params.top_k and cfg.on_device_sampling_config.global_topk and \
                params.top_k > cfg.on_device_sampling_config.global_topk:
            raise ValueError(f"top_k={params.top_k} exceeds the on-device sampler's global_topk="
                             f"{cfg.on_device_sampling_config.global_topk}")

    def abort_request(self, request_id: str):
        req = self.scheduler.requests.get(request_id)
        self.scheduler.abort_request(request_id)
        if req is not None and req.num_pending == 0 and req.slot >= 0:
            self._free_slots.append(req.slot)
            req.slot = -1

    def _watch_device_status(self):
        """Every step: raise if the status word copied (asynchronously, into pinned memory) after
        an earlier step shows an expired bounded device wait, then queue the next copy.  A kernel
        whose wait expired returns without its result, so serving stops at once instead of
        continuing on garbage (or at one expired wait per launch)."""
        from ..ops._ext import ext

        host = getattr(self, "_status_host", None)
        if host is None:
            host = self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        elif int(host[0]) != 0:
            self._check_device_status()
        ext().status_copy_async(host)

    def _check_device_status(self):
        """Raise if a bounded device wait (peer flag of a fused collective) has expired."""
        from ..ops._ext import ext

        code = int(ext().read_status())
        if code != 0:
            raise DeviceStatusError(code, f"engine step {self.num_steps}")

    @torch.no_grad()
    def prompt_hidden(self, prompts: list[list[int]]) -> torch.Tensor:
        """Final-norm hidden state of the last prompt position of each prompt ``[N, H]`` fp32
        (pooling / embedding models)."""
        return self.prompt_logits(prompts, hidden=True)

    @torch.no_grad()
    def prompt_logits(self, prompts: list[list[int]], hidden: bool = False) -> torch.Tensor:
        """Logits of the last prompt position of each prompt (one prefill step, nothing is
        sampled or kept): the hook of the logit-validation tooling.  Returns ``[N, V]`` fp32 on
        the CPU.  Must be called with no requests in flight."""
        if getattr(self.model, "dpcol", None) is not None:
            raise NotImplementedError("prompt_logits: component-DP replicas only step in lockstep (generate)")
        from .scheduler import ScheduledRequest, SchedulerOutput

        if self.has_unfinished_requests():
            raise RuntimeError("prompt_logits needs an idle engine")
        reqs = []
        try:
            for i, p in enumerate(prompts):
                r = Request(f"logits-{i}", list(p), SamplingParams(max_tokens=1))
                r.slot = self._free_slots.pop()
                if not self.block_manager.allocate(r, len(p)):
                    raise RuntimeError("not enough KV blocks for prompt_logits")
                reqs.append(r)
            out = SchedulerOutput([ScheduledRequest(r, 0, r.num_prompt_tokens, True) for r in reqs],
                                  sum(r.num_prompt_tokens for r in reqs))
            return self.runner.forward_logits(out, hidden=hidden).float().cpu()
        finally:
            for r in reqs:
                self.block_manager.free_request(r)
                self._free_slots.append(r.slot)

    # ---------------------------------------------------------------- disaggregated prefill
    def _send_remote(self, req: Request):
        """Hand a finished request to the decode engine: its tokens and the KV of every token
        but the last (whose KV the decode engine computes in its first step).  The blocks were
        just freed by the scheduler; no later step has been scheduled onto them yet."""
        bs = self.args.block_size
        n_kv = req.num_tokens - 1
        blocks = getattr(req, "freed_block_ids", req.block_ids)[:(n_kv + bs - 1) // bs]
        kv = self.kv_connector.gather_kv(self.model.kv_caches, blocks)
        meta = {"request_id": req.request_id, "prompt_token_ids": req.prompt_token_ids,
                "output_token_ids": list(req.output_token_ids), "num_kv_tokens": n_kv}
        self.kv_connector.send_request(meta, kv)

    def recv_remote(self, params=None) -> Request:
        """Receive one request from the prefill engine, install its KV into this engine's cache
        and continue it as a running decode.  ``params``: the decode's SamplingParams, or a
        callable (or dict) giving them from the request id.  Returns the request (already
        finished when the prefill engine's tokens reached a stop condition)."""
        meta, kv = self.kv_connector.recv_request(self.device)
        if isinstance(params, dict):
            params = params.get(meta["request_id"])
        elif callable(params):
            params = params(meta["request_id"])
        params = SamplingParams.coerce(params)
        req = Request(meta["request_id"], list(meta["prompt_token_ids"]), params, eos_token_id=self.eos_token_id)
        req.output_token_ids = list(meta["output_token_ids"])
        n_kv = int(meta["num_kv_tokens"])
        if not self._free_slots:
            raise RuntimeError("too many unfinished requests for the device token slots")
        if not self.block_manager.allocate(req, n_kv):
            raise RuntimeError("not enough free KV blocks for a transferred request")
        self.kv_connector.scatter_kv(self.model.kv_caches, req.block_ids, kv)
        req.num_computed_tokens = n_kv
        now = time.perf_counter()
        req.first_token_time = now
        if req.check_stop(self.max_model_len):
            req.finish_time = now
            self.block_manager.free_request(req)
            return req
        req.slot = self._free_slots.pop()
        req.status = RequestStatus.RUNNING
        self.scheduler.requests[req.request_id] = req
        self.scheduler.running.append(req)
        return req

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished() or self._inflight is not None

    # ---------------------------------------------------------------- stepping
    def _process(self, out, handle) -> list[Request]:
        toks, lps = handle.result()
        if envs.VLLM_B200_DEBUG_MODE and self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
            self._check_device_status()
        elif self.device.type == "cuda":
            self._watch_device_status()
        now = time.perf_counter()
        finished = self.scheduler.update(out, toks, lps, now=now)
        cs = getattr(self.model, "capture", None)
        for req in finished:
            if cs is not None and cs.capture is not None:
                cs.capture.save(req.request_id)
            if req.slot >= 0 and req.num_pending == 0:
                self._free_slots.append(req.slot)
                req.slot = -1
            if self.kv_connector is not None and self.kv_transfer.is_producer:
                self._send_remote(req)
        # requests that stopped earlier and just received their last in-flight token
        for s in out.scheduled:
            r = s.req
            if r.status.finished and r.num_pending == 0 and r.slot >= 0:
                self._free_slots.append(r.slot)
                r.slot = -1
        return finished

    # ---------------------------------------------------------------- profiling
    def start_profile(self, out_dir: str | None = None):
        """Start a device + host profile (torch.profiler with CUDA activities); ``stop_profile``
        writes a Chrome trace under ``out_dir`` (env ``VLLM_B200_PROFILE_DIR`` by default).
        Counterpart of the reference's /start_profile hook (NeuronProfiler,
        vllm_neuron/vllm/worker/neuron_profiler.py:38-110)."""
        import os

        from torch.profiler import ProfilerActivity, profile

        self._profile_dir = out_dir or envs.VLLM_B200_PROFILE_DIR
        acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if self.device.type == "cuda" else [])
        self._profiler = profile(activities=acts, record_shapes=False)
        self._profiler.__enter__()

    def stop_profile(self) -> str | None:
        import os

        prof = getattr(self, "_profiler", None)
        if prof is None:
            return None
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        prof.__exit__(None, None, None)
        os.makedirs(self._profile_dir, exist_ok=True)
        rank = self.tp.rank
        path = os.path.join(self._profile_dir, f"trace_rank{rank}_{int(time.time())}.json")
        prof.export_chrome_trace(path)
        self._profiler = None
        return path

    # ---------------------------------------------------------------- structured outputs
    def structured_outputs(self):
        """The grammar manager (created on first use from the tokenizer, or from
        ``self.structured_vocab`` when the engine runs on token ids only)."""
        if self._structured is None:
            from .structured import StructuredOutputManager

            eos = [self.eos_token_id] if self.eos_token_id is not None else None
            self._structured = StructuredOutputManager(self.arch.vocab_size, tokenizer=self.tokenizer,
                                                       vocab=self.structured_vocab, stop_token_ids=eos)
        return self._structured

    def _structured_step(self) -> list[Request]:
        """Synchronous step with grammar bitmasks for the requests that have one."""
        finished = []
        if self._inflight is not None:
            finished += self._process(*self._inflight)
            self._inflight = None
        out = self.scheduler.schedule()
        if out.empty:
            return finished
        samplers = [s.req for s in out.scheduled if s.samples]
        mask = self.structured_outputs().bitmask([getattr(r, "matcher", None) for r in samplers])
        before = {r.request_id: len(r.output_token_ids) for r in samplers}
        want_lp = any(r.sampling_params.logprobs for r in samplers)
        handle = self.runner.launch(out, want_logprobs=want_lp, bitmask=mask)
        self.num_steps += 1
        self.metrics.steps += 1
        finished += self._process(out, handle)
        now = time.perf_counter()
        for r in samplers:
            m = getattr(r, "matcher", None)
            if m is None or len(r.output_token_ids) == before[r.request_id]:
                continue
            for tok in r.output_token_ids[before[r.request_id]:]:
                if not m.is_terminated():
                    m.accept_token(int(tok))
            if m.is_terminated() and not r.status.finished:
                self.scheduler.finish_request(r, RequestStatus.FINISHED_STOPPED, now)
                r.stop_reason = "grammar"
                finished.append(r)
                if r.slot >= 0 and r.num_pending == 0:
                    self._free_slots.append(r.slot)
                    r.slot = -1
        return finished

    # ---------------------------------------------------------------- speculative decoding
    def _make_proposer(self, cfg: dict):
        method = cfg.get("method", "ngram")
        k = int(cfg.get("num_speculative_tokens", 3))
        if method in ("ngram", "prompt_lookup"):
            from ..spec_decode import NgramProposer

            return NgramProposer(k, cfg.get("prompt_lookup_min", 1), cfg.get("prompt_lookup_max", 4))
        if method in ("eagle3", "eagle"):
            from ..spec_decode.eagle import Eagle3Proposer

            return Eagle3Proposer(self, cfg, k)
        raise ValueError(f"unknown speculative method {method!r}")

    def _spec_step(self) -> list[Request]:
        """One synchronous step with draft verification: drafts for the decoding requests, one
        forward over [last token, drafts] (plus any prefill chunks), rejection sampling."""
        from ..spec_decode import rejection_sample

        decoding = [r for r in self.scheduler.running
                    if r.num_pending == 0 and r.num_computed_tokens == r.num_tokens - 1]
        props = self.proposer.propose(decoding) if decoding else {}
        for r in decoding:
            r.spec_token_ids = props.get(r.request_id, [])
        out = self.scheduler.schedule()
        for r in decoding:
            r.spec_token_ids = []
        if out.empty:
            return []
        self.num_steps += 1
        self.metrics.steps += 1
        logits = self.runner.forward_logits(out)
        samplers = [s for s in out.scheduled if s.samples]
        drafts = [list(s.spec) for s in samplers]
        temps = [0.0 if s.req.sampling_params.greedy else s.req.sampling_params.temperature for s in samplers]
        gens = []
        for s in samplers:
            sp = s.req.sampling_params
            g = None
            if not sp.greedy:
                g = torch.Generator()
                g.manual_seed(((sp.seed if sp.seed is not None else hash(s.req.request_id) & 0xFFFFFFFF)
                               * 1000003 + len(s.req.output_token_ids)) & 0x7FFFFFFFFFFFFFFF)
            gens.append(g)
        toks = rejection_sample(logits, drafts, temps, gens)
        if hasattr(self.proposer, "observe"):
            self.proposer.observe(out, toks)
        self.metrics.spec_draft_tokens += sum(len(d) for d in drafts)
        self.metrics.spec_accepted_tokens += sum(len(t) - 1 for t, d in zip(toks, drafts) if d)
        finished = self.scheduler.update_spec(out, toks, now=time.perf_counter())
        for req in finished:
            if hasattr(self.proposer, "release"):
                self.proposer.release(req.request_id)
            if req.slot >= 0:
                self._free_slots.append(req.slot)
                req.slot = -1
        return finished

    def step(self) -> list[Request]:
        """Schedule and launch the next step; with asynchronous scheduling the results of the
        previous step are processed while this one runs on the GPU."""
        if self.monitor is not None:
            # a peer that left (or went silent) is reported before this step launches
            now = time.perf_counter()
            if now - self._last_peer_check >= self.monitor.interval:
                self._last_peer_check = now
                self.monitor.check()
            else:
                self.monitor.check_fast()
        if self.proposer is not None:
            return self._spec_step()
        if self._has_structured and any(getattr(r, "matcher", None) is not None
                                        for r in self.scheduler.requests.values()):
            return self._structured_step()
        out = self.scheduler.schedule()
        handle = None
        if not out.empty:
            want_lp = any(s.req.sampling_params.logprobs for s in out.scheduled if s.samples)
            handle = self.runner.launch(out, want_logprobs=want_lp)
            self.num_steps += 1
            self.metrics.steps += 1
        finished = []
        if not self.async_scheduling:
            if handle is not None:
                finished = self._process(out, handle)
            return finished
        if self._inflight is not None:
            finished = self._process(*self._inflight)
            self._inflight = None
        if handle is not None:
            self._inflight = (out, handle)
        return finished

    def run_until_done(self) -> list[Request]:
        done = []
        while self.scheduler.has_unfinished() or self._inflight is not None:
            done.extend(self.step())
        return done

    def run_lockstep(self, group) -> list[Request]:
        """Serve this replica's requests in lockstep with the other data-parallel replicas of
        ``group`` (gloo): every iteration all replicas agree (MAX all-reduce of two flags and the
        batch sizes) on whether any of them has a batch and on the largest batch (the row padding
        of component data parallelism); a replica with nothing scheduled then runs a one-token
        dummy forward so that the collectives inside the model (all-to-all expert exchange)
        match.  Synchronous scheduling only.  Reference: the DP padding all-reduce and dummy
        batch (vllm_neuron/vllm/worker/neuron_model_runner.py:7337-7489, 7710)."""
        import torch.distributed as dist

        done = []
        while True:
            out = self.scheduler.schedule()
            flags = torch.tensor([0 if out.empty else 1, 1 if self.scheduler.has_unfinished() else 0,
                                  0 if out.empty else out.num_tokens,
                                  0 if out.empty else sum(s.num_logits for s in out.scheduled)],
                                 dtype=torch.int64)
            dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=group)
            # component data parallelism: every replica pads its rows to the largest batch
            self.model.dp_tmax = max(1, int(flags[2]))
            self.model.dp_smax = max(1, int(flags[3]))
            if flags[0] == 0:
                if flags[1] == 0:
                    return done
                continue
            if out.empty:
                self.runner.dummy_forward()
                continue
            want_lp = any(s.req.sampling_params.logprobs for s in out.scheduled if s.samples)
            handle = self.runner.launch(out, want_logprobs=want_lp)
            self.num_steps += 1
            self.metrics.steps += 1
            done.extend(self._process(out, handle))

    @staticmethod
    def to_output(req: Request) -> RequestOutput:
        reason = {RequestStatus.FINISHED_STOPPED: "stop", RequestStatus.FINISHED_LENGTH: "length",
                  RequestStatus.FINISHED_ABORTED: "abort"}.get(req.status)
        m = {"arrival_time": req.arrival_time, "first_token_time": req.first_token_time,
             "finish_time": req.finish_time, "num_cached_tokens": req.num_cached_tokens}
        return RequestOutput(req.request_id, req.prompt_token_ids,
                             [CompletionOutput(0, list(req.output_token_ids),
                                               logprobs=req.output_logprobs or None,
                                               finish_reason=reason)],
                             req.status.finished, m)

    def shutdown(self):
        if self.monitor is not None:
            self.monitor.stop(announce_exit=True)
        self.runner.release_graphs()
