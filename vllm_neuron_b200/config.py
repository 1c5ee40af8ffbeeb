"""Model and framework configuration.

``ModelArchConfig`` normalises a HuggingFace ``config.json`` (Llama-3, Qwen3, GPT-OSS, Qwen3
hybrid) into the fields the models use.  ``B200Config`` parses the plugin options that
users pass as ``additional_config={"neuron_config": {...}}`` (the reference's key names are
accepted verbatim, ``"b200_config"`` is an alias) -- reference:
vllm_neuron/model/neuron_config.py:8-485.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any


@dataclass
class ModelArchConfig:
    model_type: str = "llama"
    architectures: tuple = ("LlamaForCausalLM",)
    hidden_size: int = 4096
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    vocab_size: int = 128256
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None
    partial_rotary_factor: float = 1.0
    max_position_embeddings: int = 8192
    tie_word_embeddings: bool = False
    qk_norm: bool = False
    attention_bias: bool = False
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    norm_topk_prob: bool = True
    # sliding window / sinks (GPT-OSS)
    sliding_window: int = 0
    layer_types: tuple = ()
    attention_sinks: bool = False
    swiglu_limit: float = 7.0
    swiglu_alpha: float = 1.702
    # hybrid linear attention (Qwen3-Next style)
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 0
    linear_value_head_dim: int = 0
    linear_conv_kernel_dim: int = 0
    full_attention_interval: int = 0
    attn_output_gate: bool = False
    # quantization
    quant_method: str | None = None
    weight_block_size: tuple | None = None
    raw: dict = field(default_factory=dict, repr=False)

    @classmethod
    def from_hf(cls, cfg: dict) -> "ModelArchConfig":
        if hasattr(cfg, "to_dict"):
            cfg = cfg.to_dict()
        cfg = dict(cfg)
        if "text_config" in cfg and cfg.get("model_type", "").endswith("_vl"):
            text = dict(cfg["text_config"])
            text.setdefault("architectures", cfg.get("architectures"))
            cfg = {**cfg, **text}
        H = cfg.get("hidden_size", 4096)
        nh = cfg.get("num_attention_heads", 32)
        head_dim = cfg.get("head_dim") or H // nh
        qcfg = cfg.get("quantization_config") or {}
        # transformers >= 5 keeps theta and scaling under "rope_parameters"; older configs
        # use top-level "rope_theta" / "rope_scaling".
        rp = cfg.get("rope_parameters") or {}
        rope_theta = cfg.get("rope_theta", rp.get("rope_theta", 10000.0))
        rope_scaling = cfg.get("rope_scaling")
        if rope_scaling is None and rp and rp.get("rope_type", "default") != "default":
            rope_scaling = dict(rp)
        c = cls(
            model_type=cfg.get("model_type", "llama"),
            architectures=tuple(cfg.get("architectures") or ("LlamaForCausalLM",)),
            hidden_size=H,
            num_layers=cfg.get("num_hidden_layers", 32),
            num_heads=nh,
            num_kv_heads=cfg.get("num_key_value_heads", nh),
            head_dim=head_dim,
            intermediate_size=cfg.get("intermediate_size", 4 * H),
            vocab_size=cfg.get("vocab_size", 32000),
            rms_norm_eps=cfg.get("rms_norm_eps", 1e-5),
            rope_theta=rope_theta,
            rope_scaling=rope_scaling,
            partial_rotary_factor=cfg.get("partial_rotary_factor", rp.get("partial_rotary_factor", 1.0)),
            max_position_embeddings=cfg.get("max_position_embeddings", 8192),
            tie_word_embeddings=cfg.get("tie_word_embeddings", False),
            qk_norm=(cfg.get("model_type", "") in ("qwen3", "qwen3_moe", "qwen3_next", "qwen3_vl", "qwen3_vl_text",
                                                   "qwen3_5_moe", "qwen3_5_moe_text", "qwen3_5", "qwen3_5_text")
                     or bool(cfg.get("use_qk_norm", False))),
            attention_bias=cfg.get("attention_bias", cfg.get("qkv_bias",
                                                              cfg.get("model_type") in ("qwen2", "qwen2_moe"))),
            num_experts=(cfg.get("num_local_experts") or cfg.get("num_experts")
                         or cfg.get("n_routed_experts") or 0),
            num_experts_per_tok=cfg.get("num_experts_per_tok", cfg.get("experts_per_token", 0)) or 0,
            moe_intermediate_size=cfg.get("moe_intermediate_size", 0) or 0,
            shared_expert_intermediate_size=cfg.get("shared_expert_intermediate_size", 0) or 0,
            norm_topk_prob=cfg.get("norm_topk_prob", True),
            sliding_window=cfg.get("sliding_window") or 0,
            layer_types=tuple(cfg.get("layer_types") or ()),
            attention_sinks=cfg.get("model_type") == "gpt_oss",
            swiglu_limit=cfg.get("swiglu_limit", 7.0),
            linear_num_key_heads=cfg.get("linear_num_key_heads", 0) or 0,
            linear_num_value_heads=cfg.get("linear_num_value_heads", 0) or 0,
            linear_key_head_dim=cfg.get("linear_key_head_dim", 0) or 0,
            linear_value_head_dim=cfg.get("linear_value_head_dim", 0) or 0,
            linear_conv_kernel_dim=cfg.get("linear_conv_kernel_dim", 0) or 0,
            full_attention_interval=cfg.get("full_attention_interval", 0) or 0,
            attn_output_gate=cfg.get("attn_output_gate", cfg.get("model_type") == "qwen3_next"),
            quant_method=qcfg.get("quant_method"),
            weight_block_size=tuple(qcfg["weight_block_size"]) if qcfg.get("weight_block_size") else None,
            raw=cfg,
        )
        if c.model_type == "gpt_oss":
            c.intermediate_size = cfg.get("intermediate_size", c.intermediate_size)
            c.attention_bias = True
        return c

    @classmethod
    def from_path(cls, path: str) -> "ModelArchConfig":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_hf(json.load(f))

    @property
    def rot_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def layer_is_sliding(self, i: int) -> bool:
        if self.layer_types:
            return self.layer_types[i] == "sliding_attention"
        return False

    def layer_is_linear(self, i: int) -> bool:
        if self.layer_types:
            return self.layer_types[i] == "linear_attention"
        if self.full_attention_interval:
            return (i + 1) % self.full_attention_interval != 0
        return False


# -------------------------------------------------------------------------------------------
# Framework options (reference NeuronConfig keys accepted verbatim)
# -------------------------------------------------------------------------------------------
@dataclass
class OnDeviceSamplingConfig:
    """Reference: vllm_neuron/model/neuron_config.py:8-37 (enabled by default)."""

    enabled: bool = True
    do_sample: bool = True
    global_topk: int = 256
    deterministic: bool = False
    dynamic: bool = True


@dataclass
class B200Config:
    """Options under ``additional_config["neuron_config"]`` (or ``"b200_config"``)."""

    ep_degree: int | None = None
    attention_dp_size: int = 1
    embedding_dp_size: int = 1
    lm_head_dp_size: int = 1
    mlp_dp_size: int = 1
    on_device_sampling_config: OnDeviceSamplingConfig = field(default_factory=OnDeviceSamplingConfig)
    max_logprobs: int = 0
    tensor_capture: dict | None = None
    tensor_replacement: dict | None = None
    kv_segment_size_buckets: list | None = None
    debug_logits_dir: str | None = None
    quantization: str | None = None
    all2all_backend: str | None = None
    modules_to_not_convert: list | None = None
    num_batched_tokens_buckets: list | None = None
    num_seqs_buckets: list | None = None
    decode_context_length_buckets: list | None = None
    enable_structured_outputs: bool = True
    fp8_packed_kv: bool = False
    # B200-specific knobs
    sequence_parallel: bool = False   # prefill: reduce-scatter / all-gather instead of all-reduce
    cuda_graphs: bool = True
    fused_comm: bool = True           # fused GEMM+collective kernels (else NCCL baseline)
    fused_sp: bool = False            # sequence-parallel prefill on the fused RS/AG GEMMs (else NCCL)
    use_cublas_baseline: bool = False  # library GEMMs instead of the tcgen05 kernels
    # decode-size block-FP8 projections: "fp8" quantizes activations per token and 128-wide k
    # block (W8A8 on the tensor cores), "bf16" keeps them exact (W8A16)
    fp8_block_activations: str = "fp8"
    sampling_dp: bool = False          # TP decode: each rank samples 1/W of the rows (all-to-all)
    vision_tp_size: int = 1            # vision encoder sharded over this many consecutive TP ranks
    extra: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict | None) -> "B200Config":
        d = dict(d or {})
        known = {f.name for f in dataclasses.fields(cls)}
        kw: dict[str, Any] = {}
        extra = {}
        for k, v in d.items():
            if k == "on_device_sampling_config":
                if v is None:
                    kw[k] = OnDeviceSamplingConfig(enabled=False)
                elif isinstance(v, dict):
                    kw[k] = OnDeviceSamplingConfig(**v)
                else:
                    kw[k] = v
            elif k in known:
                kw[k] = v
            else:
                extra[k] = v
        c = cls(**kw)
        c.extra = extra
        c.validate()
        return c

    @classmethod
    def from_additional_config(cls, additional: dict | None) -> "B200Config":
        additional = additional or {}
        d = additional.get("b200_config") or additional.get("neuron_config") or {}
        return cls.from_dict(d)

    def validate(self):
        for name in ("attention_dp_size", "embedding_dp_size", "lm_head_dp_size", "mlp_dp_size",
                     "vision_tp_size"):
            v = getattr(self, name)
            if not isinstance(v, int) or v < 1:
                raise ValueError(f"{name} must be a positive integer, got {v!r}")
        for name in ("num_batched_tokens_buckets", "num_seqs_buckets", "decode_context_length_buckets",
                     "kv_segment_size_buckets"):
            v = getattr(self, name)
            if v is not None:
                if not all(isinstance(x, int) and x > 0 for x in v):
                    raise ValueError(f"{name} must be a list of positive integers")
                setattr(self, name, sorted(set(v)))
        if self.fp8_block_activations not in ("fp8", "bf16"):
            raise ValueError(f"fp8_block_activations must be 'fp8' or 'bf16', got {self.fp8_block_activations!r}")
        if self.all2all_backend not in (None, "neuron", "nvlink", "nccl"):
            raise ValueError(f"unknown all2all_backend {self.all2all_backend!r}")
        if self.quantization not in (None, "fp8", "fp8_static", "fp8_block", "mxfp4", "mxfp8",
                                     "modelopt_fp8", "bf16", "none"):
            raise ValueError(f"unknown quantization {self.quantization!r}")
        # Options of the reference this framework does not implement are refused rather than
        # silently ignored, so a migrated configuration never changes meaning quietly.
        if self.fp8_packed_kv:
            raise NotImplementedError("fp8_packed_kv: the packed FP8 K layout is not implemented; "
                                      "use kv_cache_dtype='fp8' (e4m3 K/V, unpacked)")
        if self.kv_segment_size_buckets is not None:
            raise NotImplementedError(
                "kv_segment_size_buckets: KV segments are not bucketed here (the decode kernel "
                "splits each sequence's KV on the device by its real length); remove the option")
        if self.decode_context_length_buckets is not None:
            raise NotImplementedError(
                "decode_context_length_buckets: decode graphs are captured per batch-size bucket "
                "and the split-KV factor follows each step's real context lengths on the device; "
                "remove the option")
        if not self.on_device_sampling_config.enabled:
            raise NotImplementedError("on_device_sampling_config=None: sampling always runs on the "
                                      "device here (logits never leave the GPU)")
        if self.max_logprobs < 0:
            raise ValueError("max_logprobs must be >= 0")
        if self.modules_to_not_convert is not None and not all(isinstance(m, str) for m in self.modules_to_not_convert):
            raise ValueError("modules_to_not_convert must be a list of module names")


@dataclass
class VisionConfig:
    """Options of the vision encoder, ``additional_config["vision_neuron_config"]``.

    ``vision_attention_block_size`` rows per packed block (images packed first-fit decreasing,
    attention restricted to each image's frames); ``num_vision_tokens_buckets`` the packed
    sizes a request's vision tokens are rounded up to (one CUDA graph of the encoder per
    bucket); default: powers of two from one block up to ``max_vision_seq_len``.
    ``tp_size`` / ``dp_size``: vision tensor parallelism over consecutive ranks and the number
    of replicas that split a request's blocks (``tp_size * dp_size`` = the TP world; the one
    left at 1 is derived).  ``encoder_cache_num_blocks``: vision encodings kept for reuse.

    Reference: vllm_neuron/model/neuron_config.py (``VisionNeuronConfig``: the same keys,
    ``resolve_tp_dp``), vllm_neuron/vllm/worker/neuron_model_runner.py:456-466.
    """

    num_vision_tokens_buckets: list | None = None
    vision_attention_block_size: int = 2048
    tp_size: int = 1
    dp_size: int = 1
    max_vision_seq_len: int | None = None
    encoder_cache_num_blocks: int | None = None
    encoder_cache_min_hold_time_ms: float | None = None
    cuda_graphs: bool = True   # capture the packed encoder per bucket

    KEY = "vision_neuron_config"

    @classmethod
    def from_dict(cls, d: dict) -> "VisionConfig":
        known = {f.name for f in dataclasses.fields(cls)}
        bad = sorted(k for k in d if k not in known)
        if bad:
            raise ValueError(f"unknown vision_neuron_config keys {bad} (known: {sorted(known)})")
        c = cls(**d)
        c.validate()
        return c

    @classmethod
    def from_additional_config(cls, additional: dict | None) -> "VisionConfig | None":
        d = (additional or {}).get(cls.KEY)
        return None if d is None else cls.from_dict(dict(d))

    def validate(self):
        bs = self.vision_attention_block_size
        if not isinstance(bs, int) or bs < 4 or bs % 4:
            raise ValueError(f"vision_attention_block_size must be a positive multiple of 4, got {bs!r}")
        for name in ("tp_size", "dp_size"):
            v = getattr(self, name)
            if not isinstance(v, int) or v < 1:
                raise ValueError(f"vision {name} must be a positive integer, got {v!r}")
        if self.max_vision_seq_len is None:
            self.max_vision_seq_len = bs
        if not isinstance(self.max_vision_seq_len, int) or self.max_vision_seq_len < 1:
            raise ValueError("max_vision_seq_len must be a positive integer")
        if self.num_vision_tokens_buckets is not None:
            b = self.num_vision_tokens_buckets
            if not b or not all(isinstance(x, int) and x > 0 for x in b):
                raise ValueError("num_vision_tokens_buckets must be a non-empty list of positive integers")
            self.num_vision_tokens_buckets = sorted(set(b))
        else:
            top = max(bs, -(-self.max_vision_seq_len // bs) * bs)
            b, n = [], bs
            while n < top:
                b.append(n)
                n *= 2
            self.num_vision_tokens_buckets = b + [top]
        if self.encoder_cache_num_blocks is not None and (
                not isinstance(self.encoder_cache_num_blocks, int) or self.encoder_cache_num_blocks < 1):
            raise ValueError("encoder_cache_num_blocks must be a positive integer")

    def resolve_tp_dp(self, world: int) -> tuple[int, int]:
        """Concrete (vision TP, vision DP) for a TP world of ``world`` ranks."""
        tp, dp = self.tp_size, self.dp_size
        if tp == 1 and dp == 1:
            tp, dp = 1, world
        elif dp == 1:
            dp = world // tp
        elif tp == 1:
            tp = world // dp
        if tp * dp != world or tp < 1 or dp < 1:
            raise ValueError(f"vision tp_size {self.tp_size} x dp_size {self.dp_size} does not "
                             f"match the world of {world} ranks")
        self.tp_size, self.dp_size = tp, dp
        return tp, dp


def vision_tp_of(additional: dict | None) -> int:
    """Vision TP degree from either the vision config (``tp_size``) or ``vision_tp_size`` of the
    framework options (they must agree when both are given)."""
    a = additional or {}
    opts = a.get("neuron_config") or a.get("b200_config") or {}
    legacy = int(opts.get("vision_tp_size", 1))
    vd = a.get(VisionConfig.KEY) or {}
    vt = int(vd.get("tp_size", 1))
    if legacy > 1 and vt > 1 and legacy != vt:
        raise ValueError(f"vision_tp_size={legacy} and vision_neuron_config.tp_size={vt} disagree")
    return max(legacy, vt)
