"""Llama-3 / Qwen3 dense decoder on the sm_100a kernels, tensor parallel over a GroupComm.

Per layer (TP world W, local heads Hq/W and Hkv/W, local FFN I/W):

  prefill / mixed batches (tokens > 128):
    qkv  = x @ Wqkv^T                         tcgen05 GEMM, bf16 out
    q, k/v -> cache                           rope_kv_write (RoPE, optional QK-norm)
    a    = paged_attention(q, cache)
    o    = a @ Wo^T  -> all-reduce (W > 1)    row-parallel
    x    = rmsnorm(residual += o)
    act  = silu(x @ Wg^T) * (x @ Wu^T)        one GEMM with the SwiGLU epilogue
    d    = act @ Wd^T -> all-reduce
    x    = rmsnorm(residual += d)             (the next layer's input norm)

  decode batches (tokens <= 128): the same with swapped-operand split-K GEMMs that
  accumulate in fp32 buffers; the consumer kernels read and clear those buffers, and the
  all-reduce (W > 1) runs on the fp32 buffer.

Weights: ``qkv [(Hq + 2 Hkv) D / W, H]``, ``o [H, Hq D / W]``, ``gate_up`` rows interleaved
in 128-row blocks ``[2 I / W, H]``, ``down [H, I / W]``, vocab-sharded embedding and LM head.

Reference: vllm_neuron/model/llama3/model.py (LlamaAttention :333-991, LlamaMLP
:1017-1115, LlamaModel.forward :1424, LlamaForCausalLM.forward :1610) and
vllm_neuron/model/qwen3/model.py (QK-norm).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import ops
from ..config import ModelArchConfig
from ..ops import linear as L
from ..parallel.comm import SINGLE, GroupComm


@dataclass
class ForwardBatch:
    """Device-side inputs of one forward pass (built by the model runner)."""

    input_ids: torch.Tensor      # [T] int32
    positions: torch.Tensor      # [T] int32
    slot_mapping: torch.Tensor   # [T] int32 (-1 = do not write)
    block_tables: torch.Tensor   # [B, max_blocks] int32
    seq_lens: torch.Tensor       # [B] int32
    q_start: torch.Tensor        # [B + 1] int32
    work: torch.Tensor           # [W, 2] int32 attention work items
    logits_indices: torch.Tensor  # [S] int64 rows whose logits are needed
    decode: bool
    num_splits: int
    num_tokens: int
    last_tok: torch.Tensor | None = None  # device-resident tokens for ids < 0
    seq_slots: torch.Tensor | None = None  # [B] int32 per-request state-cache slots
    want_hidden: bool = False  # return the final-norm hidden states of the logits rows (pooling)
    embed_rows: torch.Tensor | None = None   # [n] int64 batch rows whose embeddings are given
    embeds: torch.Tensor | None = None       # [n, H] the given embeddings (prompt_embeds)
    positions3: torch.Tensor | None = None   # [T, 3] int32 M-RoPE positions (vision-language)
    deep_rows: torch.Tensor | None = None    # [n] int64 rows receiving DeepStack features
    deep_feats: torch.Tensor | None = None   # [n_deep, n, H] added after decoder layers 0..n_deep-1
    max_q_len: int = 0                       # longest query of the step (host value; 0 = unknown)
    splits_dev: torch.Tensor | None = None   # [1] int32 split-KV factor of this decode step
    seq_lens_local: torch.Tensor | None = None  # [B] int32 tokens held by this DCP rank
    prefill_rows: int = 64                   # packed query rows per prefill work item (64 / 128)


def _shard(n: int, world: int, rank: int) -> tuple[int, int]:
    assert n % world == 0, f"{n} not divisible by TP={world}"
    per = n // world
    return rank * per, per


class LlamaForCausalLM(torch.nn.Module):
    """Dense Llama-3 / Qwen3 decoder (the ``LlamaForCausalLM`` / ``Qwen3ForCausalLM`` archs)."""
    supports_dcp = True  # decode context parallelism (token-sharded KV)

    def __init__(self, cfg: ModelArchConfig, tp: GroupComm = SINGLE, device="cuda",
                 dtype=torch.bfloat16, max_tokens: int = 8192, max_decode_tokens: int = 128,
                 max_seqs: int = 256, block_size: int = 16):
        super().__init__()
        self.cfg = cfg
        self.tp = tp
        self.device = torch.device(device)
        self.dtype = dtype
        W = tp.world
        self.Hq = cfg.num_heads // W
        # KV heads are replicated when TP exceeds their count.
        self.kv_rep = max(1, W // cfg.num_kv_heads)
        self.Hkv = max(1, cfg.num_kv_heads // W)
        self.D = cfg.head_dim
        self.H = cfg.hidden_size
        self.I = cfg.intermediate_size // W
        self.V = cfg.vocab_size
        self.V_local = math.ceil(cfg.vocab_size / W)
        self.vocab_start = tp.rank * self.V_local
        self.eps = cfg.rms_norm_eps
        self.scale = 1.0 / math.sqrt(self.D)
        self.silu_blk = L.SILU_BLOCK if self.I % L.SILU_BLOCK == 0 else 0
        self.block_size = block_size
        self.max_decode_tokens = max_decode_tokens
        self.max_tokens = max_tokens
        qkv_out = (self.Hq + 2 * self.Hkv) * self.D
        self.qkv_out = qkv_out
        p = lambda *s: torch.nn.Parameter(torch.empty(*s, dtype=dtype, device=self.device), requires_grad=False)
        self.embed = p(self.V_local, self.H)
        self.layers = torch.nn.ModuleList()
        for _ in range(cfg.num_layers):
            m = torch.nn.Module()
            m.input_norm = p(self.H)
            m.post_norm = p(self.H)
            self._make_attn(m, p, len(self.layers))
            self._make_mlp(m, p, len(self.layers))
            self.layers.append(m)
        self.final_norm = p(self.H)
        self.lm_head = self.embed if cfg.tie_word_embeddings else p(self.V_local, self.H)
        self.cos_sin = ops.cos_sin_table(cfg.max_position_embeddings, cfg.rot_dim, cfg.rope_theta,
                                         cfg.rope_scaling, device=self.device)
        # long-context query temperature (Ministral-3: rope_parameters.llama_4_scaling_beta)
        rp = cfg.rope_scaling or {}
        beta = rp.get("llama_4_scaling_beta")
        self.q_pos_scale = ((float(beta), float(rp.get("original_max_position_embeddings") or 8192))
                            if beta else None)
        self.kv_caches: list[tuple[torch.Tensor, torch.Tensor]] = []
        self._alloc_workspace(max_tokens, max_decode_tokens, max_seqs)
        self.tp_fused = None  # TPFusedComm: fused all-reduce + residual + RMSNorm (decode)
        self.dcp = SINGLE     # decode-context-parallel replica set (KV tokens sharded over it)
        self.sequence_parallel = False  # prefill residual stream sharded over tokens (TP > 1)
        self.mrope_section = None       # (t, h, w) frequency split of the multimodal RoPE
        self._sp = None                 # (padded tokens, local tokens) of the running SP forward
        self.sp_fused = None            # SPFusedComm: fused SP collectives (CUDA, TP > 1)
        self._spf = False               # the running forward uses sp_fused
        self.sp_forwards = 0            # forwards that ran sequence-parallel
        # Hidden states captured after these layers (EAGLE3 drafting): [tokens, len * H]
        self.aux_layers: list[int] = []
        self.aux_hidden: torch.Tensor | None = None
        # accuracy tooling: activation capture / golden replacement (accuracy.tensor_capture)
        self.capture = None
        # component data parallelism (set_component_dp): the DP column and the component TP
        # group over every replica; the step's largest replica batch (tokens / logits rows)
        self.dpcol = None
        self.comp_tp = None
        self.cdp_mlp = self.cdp_embed = self.cdp_lmh = self.cdp_attn = False
        self.lm_head_from_embed = False
        self.dp_tmax = self.dp_smax = 1

    # ---------------------------------------------------------------- init / weights
    def _make_attn(self, m, p, layer: int):
        """Attention parameters of one layer."""
        cfg = self.cfg
        m.qkv = p(self.qkv_out, self.H)
        m.qkv_bias = p(self.qkv_out) if cfg.attention_bias else None
        m.o = p(self.H, self.Hq * self.D)
        m.o_bias = None
        m.window = cfg.sliding_window if cfg.layer_is_sliding(layer) else 0
        m.sinks = None
        if cfg.qk_norm:
            m.q_norm = p(self.D)
            m.k_norm = p(self.D)
        else:
            m.q_norm = m.k_norm = None

    def _make_mlp(self, m, p, layer: int):
        """Dense SwiGLU MLP parameters of one layer (MoE models override this)."""
        m.gate_up = p(2 * self.I, self.H)
        m.down = p(self.H, self.I)

    def _alloc_workspace(self, max_tokens, max_dec, max_seqs):
        d, bf = self.device, self.dtype
        W = self.tp.world
        max_tokens = -(-max_tokens // W) * W  # sequence parallelism pads the tokens to W
        # sequence-parallel local slices (residual stream sharded over tokens)
        self.ws_sp_x = torch.zeros(max_tokens // W, self.H, dtype=bf, device=d)
        self.ws_sp_h = torch.zeros(max_tokens // W, self.H, dtype=bf, device=d)
        self.ws_residual = torch.zeros(max_tokens, self.H, dtype=bf, device=d)
        self.ws_x = torch.zeros(max_tokens, self.H, dtype=bf, device=d)
        self.ws_qkv = torch.zeros(max_tokens, self.qkv_out, dtype=bf, device=d)
        self.ws_q = torch.zeros(max_tokens, self.Hq * self.D, dtype=bf, device=d)
        self.ws_attn = torch.zeros(max_tokens, self.Hq * self.D, dtype=bf, device=d)
        self.ws_h = torch.zeros(max_tokens, self.H, dtype=bf, device=d)
        self.ws_act = torch.zeros(max_tokens, self.I, dtype=bf, device=d)
        # fp32 accumulation buffers of the decode path (kept zero between uses)
        self.acc_qkv = torch.zeros(max_dec, self.qkv_out, dtype=torch.float32, device=d)
        self.acc_h = torch.zeros(max_dec, self.H, dtype=torch.float32, device=d)
        self.acc_gu = torch.zeros(max_dec, 2 * self.I, dtype=torch.float32, device=d)
        self.ws_logits_x = torch.zeros(max_seqs, self.H, dtype=bf, device=d)
        self.ws_logits = torch.zeros(max_seqs, self.V_local, dtype=bf, device=d)
        self.attn_splits_max = 32
        self.ws_part_o = torch.zeros(self.attn_splits_max * max_dec * self.Hq * self.D,
                                     dtype=torch.float32, device=d)
        self.ws_part_lse = torch.zeros(self.attn_splits_max * max_dec * self.Hq,
                                       dtype=torch.float32, device=d)

    @torch.no_grad()
    def init_random(self, seed: int = 0, std: float = 0.02):
        """Random-init N(0, std) weights (norms = 1).  Each TP rank draws its own shard."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 1000 + self.tp.rank)
        for name, prm in self.named_parameters():
            if prm is None:
                continue
            if "norm" in name:
                prm.fill_(1.0)
            elif name.endswith("bias"):
                prm.zero_()
            else:
                prm.normal_(0.0, std, generator=g)

    def enable_fused_comm(self, cpu_group=None, fused_sp: bool = True):
        """Use the fused one-shot all-reduce + residual + RMSNorm kernel for TP decode, and with
        ``fused_sp`` (and sequence parallelism on) the fused reduce-scatter / all-gather GEMMs for
        prefill."""
        if self.tp.world > 1 and self.device.type == "cuda":
            from ..parallel.fused import TPFusedComm

            self.tp_fused = TPFusedComm(self.tp, self.H, self.max_decode_tokens, self.device, cpu_group)
            # Sequence-parallel prefill with the all-gather / reduce-scatter fused into the GEMMs
            # and the norm: dense SwiGLU decoders without an o_proj bias
            if (fused_sp and self.sequence_parallel and type(self)._mlp is LlamaForCausalLM._mlp
                    and all(getattr(ly, "o_bias", None) is None for ly in self.layers)
                    and (not getattr(self, "fp8_linears", 0) or getattr(self, "block_fp8", False))):
                from ..parallel.fused import SPFusedComm

                self.sp_fused = SPFusedComm(self.tp, self.H, self.max_tokens + self.tp.world, self.device,
                                            cpu_group)

    @property
    def num_kv_layers(self) -> int:
        return self.cfg.num_layers

    def bind_kv_cache(self, kv_caches: list[tuple[torch.Tensor, torch.Tensor]]):
        assert len(kv_caches) == self.num_kv_layers
        self.kv_caches = kv_caches
        for ly in self.layers:  # weights are final here: refresh the fp32 bias copies
            for name in ("qkv_bias", "o_bias"):
                if getattr(ly, name, None) is not None:
                    setattr(ly, name + "_f32", None)
                    self._f32(ly, name)

    def kv_cache_shape(self, num_blocks: int) -> tuple[int, ...]:
        return (num_blocks, self.Hkv, self.block_size, self.D)

    @property
    def kv_dtype(self) -> torch.dtype:
        """Element type of the KV cache: the model dtype, or ``torch.float8_e4m3fn`` after
        :meth:`set_kv_cache_dtype` ("fp8")."""
        return getattr(self, "_kv_dtype", None) or self.dtype

    def kv_scale(self, kv_layer: int) -> tuple[float, float]:
        """Per-tensor (k_scale, v_scale) of an fp8 cache layer (1.0 when not quantized)."""
        sc = getattr(self, "kv_scales", None)
        return sc[kv_layer] if sc else (1.0, 1.0)

    # components whose component / attention DP this model's forward and checkpoint loader cover
    component_dp_parts = ("mlp", "embed", "lm_head", "attn")

    # weights that block-FP8 serving quantizes (2-D linears, 3-D expert stacks); the router,
    # norms, embeddings and LM head stay bf16
    BLOCK_FP8_PARAMS = ("qkv", "o", "gate_up", "down", "w_gu", "w_down", "sh_gu", "sh_down",
                        "w_in", "out_proj", "qkvg")

    # projections of a decoder layer and the checkpoint names whose scales they take
    FP8_LINEARS = (("qkv", ("q_proj", "k_proj", "v_proj")), ("o", ("o_proj",)),
                   ("gate_up", ("gate_proj", "up_proj")), ("down", ("down_proj",)))

    @torch.no_grad()
    def quantize_fp8_static(self, scales: dict | None = None, default_in_scale: float = 1.0 / 32):
        """Switch the dense projections to static per-tensor FP8 (W8A8) on the tcgen05 FP8 GEMM.
        ``scales[(layer, proj)] = (weight_scale, input_scale)`` from the checkpoint; fused
        projections take the largest scale of their parts (requantized), and without
        checkpoint scales the weight scale is amax / 448 and the input scale
        ``default_in_scale``.  Reference: vllm_neuron/model/llama3/quantization.py:39-310."""
        n = 0
        for i, ly in enumerate(self.layers):
            for name, parts in self.FP8_LINEARS:
                w = getattr(ly, name, None)
                if w is None or isinstance(w, L.FP8Weight) or not isinstance(w, torch.Tensor):
                    continue
                ws = ins = None
                if scales:
                    got = [scales[(i, p)] for p in parts if (i, p) in scales]
                    if got:
                        ws = max(g[0] for g in got)
                        ins = max(g[1] for g in got)
                fw = L.FP8Weight.from_weight(w, ws, ins if ins is not None else default_in_scale)
                if name in getattr(ly, "_parameters", {}):
                    del ly._parameters[name]
                setattr(ly, name, fw)
                n += 1
        self.fp8_linears = n
        return n

    @torch.no_grad()
    def quantize_block_fp8(self) -> int:
        """Switch the dense projections to block-scaled FP8 weights (e4m3, one fp32 scale per
        128 x 128 block of the rank's fused shard; W8A16 on the tcgen05 GEMM).  A block-FP8
        checkpoint whose blocks align with the shard (rows and K in multiples of 128, as for
        Llama-3-70B at TP 8) is recovered exactly: its values re-quantize to the same bytes.
        Random-init weights are quantized from their bf16 draw (``quantization: fp8_block``)."""
        n = 0
        for ly in self.layers:
            for name in self.BLOCK_FP8_PARAMS:
                w = getattr(ly, name, None)
                if w is None or not isinstance(w, torch.Tensor) or w.dim() not in (2, 3):
                    continue
                if w.dim() == 3 and w.shape[1] % L.BlockFP8Weight.BLOCK:
                    continue  # stacked experts need 128-row experts
                bw = L.BlockFP8Weight.from_weight(w)
                if name in getattr(ly, "_parameters", {}):
                    del ly._parameters[name]
                setattr(ly, name, bw)
                n += 1
        self.fp8_linears = n
        self.block_fp8 = True
        if self.device.type == "cuda":
            torch.cuda.empty_cache()
        return n

    @torch.no_grad()
    def quantize_mxfp8(self) -> int:
        """Switch the dense 2-D projections (K a multiple of 128) to MXFP8 weights: e4m3 values
        with one e8m0 scale per 32 input elements, served W8A8 on the block-scaled tensor cores
        (activations quantized to MXFP8 per token on the fly); bf16 expert stacks with 128-row
        experts and K in 128s run on the grouped form of the same GEMM.  An MXFP8 checkpoint,
        loaded as its exact bf16 dequantization, re-quantizes to the same values (power-of-two
        scales).  MXFP4 expert stacks stay in their format.  Reference: the MXFP8 text decoder of Qwen3-VL
        (vllm_neuron/model/qwen3_vl/model_mxfp8.py) and the MX linears of
        vllm_neuron/model/llama3/model_mx_fp8.py."""
        n = 0
        for ly in self.layers:
            for name in self.BLOCK_FP8_PARAMS:
                w = getattr(ly, name, None)
                if w is None or not isinstance(w, torch.Tensor) or w.dim() not in (2, 3) or w.shape[-1] % 128:
                    continue
                if w.dim() == 3 and w.shape[1] % 128:
                    continue  # the grouped MXFP8 GEMM needs 128-row experts
                mw = L.MXFP8Weight.from_weight(w)
                if name in getattr(ly, "_parameters", {}):
                    del ly._parameters[name]
                setattr(ly, name, mw)
                n += 1
        self.mx_linears = n
        if self.device.type == "cuda":
            torch.cuda.empty_cache()
            # activation buffers at their largest size before any decode graph is captured
            ks = {w.shape[-1] for ly in self.layers for w in vars(ly).values()
                  if isinstance(w, L.MXFP8Weight) and w.q.dim() == 2}
            for k in ks:
                L.MX8Activations.reserve(self.max_tokens, k, self.device)
        return n

    def set_kv_cache_dtype(self, kv_cache_dtype: str, scales: list[tuple[float, float]] | None = None):
        """``"auto"`` keeps the model dtype; ``"fp8"`` / ``"fp8_e4m3"`` stores e4m3 K/V with
        per-layer scales (true value = byte * scale; default 1.0), the reference's FP8 KV
        cache (vllm_neuron/model/llama3/model.py:2150-2180)."""
        if kv_cache_dtype in (None, "auto", "bfloat16", "bf16"):
            self._kv_dtype = None
            self.kv_scales = None
            return
        if kv_cache_dtype not in ("fp8", "fp8_e4m3"):
            raise ValueError(f"unsupported kv_cache_dtype {kv_cache_dtype!r} (auto, fp8, fp8_e4m3)")
        self._kv_dtype = torch.float8_e4m3fn
        n = self.num_kv_layers
        self.kv_scales = list(scales) if scales else [(1.0, 1.0)] * n
        if len(self.kv_scales) != n:
            raise ValueError(f"expected {n} KV scale pairs, got {len(self.kv_scales)}")

    def kv_bytes_per_block(self) -> int:
        return 2 * self.num_kv_layers * self.Hkv * self.block_size * self.D * self.kv_dtype.itemsize

    # ---------------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, b: ForwardBatch) -> torch.Tensor:
        """Returns logits ``[len(logits_indices), V]`` (bf16, full vocab on every rank)."""
        T = b.num_tokens
        small = T <= self.max_decode_tokens
        fused = small and self.tp_fused is not None
        tp = self.tp
        res, x, Tg = self._embed(b, T, small)
        cs = self.capture
        if cs is not None and cs.point("model.embed_tokens", res[:T]):
            ops.rmsnorm(res[:T], self.layers[0].input_norm, self.eps, out=x[:T])
        nL = len(self.layers)
        for i, ly in enumerate(self.layers):
            k_cache, v_cache = self.kv_caches[i]
            ks, vs = self.kv_scale(i)
            if self.cdp_attn:
                self._attention_dp(ly, x, res, b, T, k_cache, v_cache, (ks, vs))
            else:
                q = self.ws_q[:T]
                # ---- attention
                if small:
                    acc = self.acc_qkv[:T]
                    L.gemm_accumulate(x, ly.qkv, acc)
                    ops.rope_kv_write(acc, b.positions, self.cos_sin, self.Hq, self.Hkv, self.D, q,
                                      k_cache, v_cache, b.slot_mapping, ly.q_norm, ly.k_norm, self.eps,
                                      rot_dim=self.cfg.rot_dim, clear_input=True, q_pos_scale=self.q_pos_scale,
                                      qkv_bias=self._f32(ly, "qkv_bias"), positions3=b.positions3,
                                      mrope_section=self.mrope_section, k_scale=ks, v_scale=vs)
                else:
                    if self._spf:
                        qkv = self.sp_fused.gemm_ag(x[:T], ly.qkv, self.ws_qkv[:T], L.EPI_BF16,
                                                    L._pick_bn_wide(T, ly.qkv.shape[0], L.num_sms(x.device)))
                    else:
                        qkv = L.gemm_out(x[:T], ly.qkv, out=self.ws_qkv[:T])
                    ops.rope_kv_write(qkv, b.positions, self.cos_sin, self.Hq, self.Hkv, self.D, q,
                                      k_cache, v_cache, b.slot_mapping, ly.q_norm, ly.k_norm, self.eps,
                                      rot_dim=self.cfg.rot_dim, q_pos_scale=self.q_pos_scale,
                                      qkv_bias=self._f32(ly, "qkv_bias"), positions3=b.positions3,
                                      mrope_section=self.mrope_section, k_scale=ks, v_scale=vs)
                attn = self.ws_attn[:T]
                self._attention(q, attn, k_cache, v_cache, b, window=ly.window, sinks=ly.sinks,
                                kv_scale=(ks, vs))
                nxt_norm = ly.post_norm
                if small:
                    acc = self.acc_h[:T]
                    L.gemm_accumulate(attn, ly.o, acc)
                    if ly.o_bias is not None and tp.rank == 0:
                        acc.add_(self._f32(ly, "o_bias"))
                    self._allreduce_norm(acc, res, nxt_norm, x, fused)
                else:
                    if Tg > T:
                        self.ws_attn[T:Tg].zero_()
                    if self._spf:
                        x = self._gemm_rs_norm(self.ws_attn[:Tg], ly.o, res, nxt_norm)
                    else:
                        h = L.gemm_out(self.ws_attn[:Tg], ly.o, out=self.ws_h[:Tg])
                        if ly.o_bias is not None and tp.rank == 0:
                            h.add_(ly.o_bias)
                        self._reduce_norm(h, res, nxt_norm, x)
            # ---- MLP
            nxt_norm = self.layers[i + 1].input_norm if i + 1 < nL else self.final_norm
            x_new = self._mlp(i, ly, x, res, nxt_norm, Tg, small, fused)
            if x_new is not None:
                x = x_new
            if b.deep_feats is not None and i < b.deep_feats.shape[0]:
                # DeepStack: visual features join the residual stream of the image-token rows
                r = b.deep_rows
                res.index_add_(0, r, b.deep_feats[i].to(res.dtype))
                x.index_copy_(0, r, ops.rmsnorm(res.index_select(0, r), nxt_norm, self.eps).to(x.dtype))
            if cs is not None and cs.point(f"model.layers.{i}", res[:T]):
                ops.rmsnorm(res[:T], nxt_norm, self.eps, out=x[:T])
            if self.aux_layers and i in self.aux_layers:
                j = self.aux_layers.index(i)
                self.aux_hidden[:T, j * self.H:(j + 1) * self.H].copy_(res)
        self._sp = None
        if self._spf:
            self._spf = False
            self.sp_fused.wait_gathered()  # the final norm's rows from every rank
            self.sp_fused.forwards += 1
        if cs is not None:
            cs.point("model.norm", x[:T])
        if b.want_hidden:
            return x.index_select(0, b.logits_indices.long())
        logits = self.compute_logits(x, b.logits_indices)
        if cs is not None:
            cs.point("lm_head", logits, logits=True)
        return logits

    def _gemm_rs_norm(self, a: torch.Tensor, w: torch.Tensor, res: torch.Tensor, norm_w: torch.Tensor) -> torch.Tensor:
        """Fused SP row-parallel epilogue: GEMM reduce-scattered into the owners' slots, then
        residual add + RMSNorm + all-gather push; returns the gathered normalized rows."""
        self.sp_fused.gemm_rs(a, w, L._pick_bn_wide(a.shape[0], w.shape[0], L.num_sms(a.device)))
        return self.sp_fused.norm_push(res, norm_w, self.eps, reduce=True)

    @staticmethod
    def _f32(ly, name: str) -> torch.Tensor | None:
        """fp32 copy of a bias parameter, cached on the layer (made at KV-cache binding, before
        any graph capture, so the forward launches no conversion kernels)."""
        t = getattr(ly, name, None)
        if t is None:
            return None
        c = getattr(ly, name + "_f32", None)
        if c is None or c.shape != t.shape:
            c = t.detach().float().contiguous()
            setattr(ly, name + "_f32", c)
        return c

    def _embed(self, b: ForwardBatch, T: int, small: bool):
        """Embedding (vocab-parallel) and the first RMSNorm.  Returns ``(res, x, Tg)``: the
        residual stream, the normalized full-token activations and the GEMM row count.

        Under sequence parallelism (TP > 1 prefill) the token count is padded to a multiple of
        the TP size ``Tg``; each rank keeps the residual rows ``[rank*Tg/W, (rank+1)*Tg/W)``
        (reduce-scatter of the embedding partial sums) and ``x`` is the all-gathered normalized
        activation of all ``Tg`` rows (reference: SP prefill, model/llama3/model.py:527-532,
        813-815,1096-1111; nn/embedding.py:236-241)."""
        tp = self.tp
        use_sp = (self.sequence_parallel and tp.world > 1 and not small and b.embed_rows is None
                  and not self.cdp_embed
                  and b.deep_feats is None and not self.aux_layers and self.capture is None)
        if not use_sp:
            self._sp = None
            res = self.ws_residual[:T]
            x = self.ws_x[:T]
            if self.cdp_embed:
                self._embed_cdp(b, res, T)
            else:
                ops.embedding(b.input_ids, self.embed, self.vocab_start, self.vocab_start + self.V_local,
                              out=res, last_tok=b.last_tok)
                tp.all_reduce_(res)
            if b.embed_rows is not None:
                res.index_copy_(0, b.embed_rows, b.embeds.to(res.dtype))
            ops.rmsnorm(res, self.layers[0].input_norm, self.eps, out=x)
            return res, x, T
        W = tp.world
        Tg = -(-T // W) * W
        Tl = Tg // W
        self._sp = (Tg, Tl)
        self.sp_forwards += 1
        full = self.ws_h[:Tg]
        ops.embedding(b.input_ids, self.embed, self.vocab_start, self.vocab_start + self.V_local,
                      out=full[:T], last_tok=b.last_tok)
        if Tg > T:
            full[T:].zero_()
        res = self.ws_residual[:Tl]
        tp.reduce_scatter(full, out=res)
        self._spf = self.sp_fused is not None and Tl <= self.sp_fused.Tl_max
        if self._spf:
            # RMSNorm + all-gather push of the local rows in one kernel
            return res, self.sp_fused.norm_push(res, self.layers[0].input_norm, self.eps, reduce=False), Tg
        x_l = self.ws_sp_x[:Tl]
        ops.rmsnorm(res, self.layers[0].input_norm, self.eps, out=x_l)
        x = self.ws_x[:Tg]
        tp.all_gather(x_l, dim=0, out=x)
        return res, x, Tg

    def _reduce_norm(self, h: torch.Tensor, res: torch.Tensor, norm_w: torch.Tensor, x: torch.Tensor):
        """Prefill row-parallel epilogue: ``res += sum_ranks(h)``; ``x = rmsnorm(res) * w``.
        All-reduce, or under sequence parallelism reduce-scatter -> local add + RMSNorm ->
        all-gather (same bytes on the wire, norms on 1/W of the rows)."""
        if self._sp is None:
            self.tp.all_reduce_(h)
            ops.add_rmsnorm(h, res, norm_w, self.eps, out=x)
            return
        Tg, Tl = self._sp
        h_l = self.ws_sp_h[:Tl]
        self.tp.reduce_scatter(h[:Tg], out=h_l)
        x_l = self.ws_sp_x[:Tl]
        ops.add_rmsnorm(h_l, res, norm_w, self.eps, out=x_l)
        self.tp.all_gather(x_l, dim=0, out=x[:Tg])

    def enable_aux_hidden(self, layers: list[int]):
        """Capture the residual stream after ``layers`` in every forward (draft models)."""
        self.aux_layers = list(layers)
        self.aux_hidden = torch.zeros(self.max_tokens, len(layers) * self.H, dtype=self.dtype,
                                      device=self.device)

    def _mlp(self, i: int, ly, x, res, nxt_norm, T: int, small: bool, fused: bool):
        """Dense SwiGLU MLP; leaves ``x = nxt_norm(res += mlp(x))``."""
        if self.cdp_mlp:
            return self._mlp_cdp(ly, x, res, nxt_norm, T)
        if small:
            acc = self.acc_gu[:T]
            L.gemm_accumulate(x, ly.gate_up, acc)
            act = ops.silu_mul(acc, out=self.ws_act[:T], blk=self.silu_blk, clear_input=True)
            acc = self.acc_h[:T]
            L.gemm_accumulate(act, ly.down, acc)
            self._allreduce_norm(acc, res, nxt_norm, x, fused)
        else:
            if self._spf:
                if self.silu_blk:
                    act = self.sp_fused.gemm_ag(x, ly.gate_up, self.ws_act[:T], L.EPI_SILU_BF16, 2 * L.SILU_BLOCK)
                else:
                    gu = torch.empty(T, ly.gate_up.shape[0], dtype=x.dtype, device=x.device)
                    self.sp_fused.gemm_ag(x, ly.gate_up, gu, L.EPI_BF16,
                                          L._pick_bn_wide(T, ly.gate_up.shape[0], L.num_sms(x.device)))
                    act = ops.silu_mul(gu, out=self.ws_act[:T])
                return self._gemm_rs_norm(act, ly.down, res, nxt_norm)
            if self.silu_blk:
                act = L.gemm_silu(x, ly.gate_up, out=self.ws_act[:T])
            else:
                gu = L.gemm_out(x, ly.gate_up)
                act = ops.silu_mul(gu, out=self.ws_act[:T])
            h = L.gemm_out(act, ly.down, out=self.ws_h[:T])
            self._reduce_norm(h, res, nxt_norm, x)

    def set_component_dp(self, groups: dict):
        """Component data parallelism over data-parallel replicas that step in lockstep: the
        chosen components (dense MLP, embedding, LM head) shard their weights over ``comp_tp``
        (every rank of every replica, TP x DP) instead of the replica's TP group.  Before such a
        component, the replicas' rows are all-gathered over ``dpcol`` (the ranks at this TP
        position in the other replicas), padded to the step's largest replica batch
        (``dp_tmax`` tokens / ``dp_smax`` logits rows); each rank computes its shard on all rows,
        ``groups`` maps each component (``"mlp"``, ``"embed"``, ``"lm_head"``, ``"attn"``) to its
        (DP column, component TP group): k replicas share a component when its size is k;
        the shards are combined over ``comp_tp`` (all-reduce, or an all-gather of vocab slices
        for the LM head) and each replica keeps its own rows.  Attention (and its KV cache of
        the replica's own requests) stays on the replica.  Call before the weights load.
        Reference: component-level DP sharding (``mlp_dp_size`` / ``embedding_dp_size`` /
        ``lm_head_dp_size``, docs/design/parallelism/component_dp_sharding.md; groups
        vllm_neuron/parallel/neuron_parallel_state.py:619-665)."""
        parts = set(self.component_dp_parts)
        if type(self)._mlp is not LlamaForCausalLM._mlp:
            parts.discard("mlp")  # expert MLPs shard by EP instead
        bad = sorted(set(groups) - parts)
        if bad:
            raise NotImplementedError(f"component data parallelism of {bad} is not supported by {type(self).__name__}")
        p = lambda *s: torch.nn.Parameter(torch.empty(*s, dtype=self.dtype, device=self.device), requires_grad=False)
        self.cdp_groups = dict(groups)
        self.dpcol, self.comp_tp = next(iter(groups.values()))  # any: marks lockstep stepping
        mlp, embed, lm_head = ("mlp" in groups), ("embed" in groups), ("lm_head" in groups)
        tied = self.lm_head is self.embed
        if mlp:
            W = groups["mlp"][1].world
            if self.cfg.intermediate_size % W:
                raise ValueError(f"the MLP width {self.cfg.intermediate_size} does not split over {W} ranks")
            self.cdp_mlp = True
            self.I = self.cfg.intermediate_size // W
            self.silu_blk = L.SILU_BLOCK if self.I % L.SILU_BLOCK == 0 else 0
            for i, ly in enumerate(self.layers):
                self._make_mlp(ly, p, i)
            self.ws_act = torch.zeros(self.ws_act.shape[0], self.I, dtype=self.dtype, device=self.device)
            self.acc_gu = torch.zeros(self.acc_gu.shape[0], 2 * self.I, dtype=torch.float32, device=self.device)
        if embed:
            cg = groups["embed"][1]
            vl = math.ceil(self.V / cg.world)
            self.cdp_embed = True
            self.V_local_emb, self.vocab_start_emb = vl, cg.rank * vl
            self.embed = p(vl, self.H)
        if lm_head:
            vl = math.ceil(self.V / groups["lm_head"][1].world)
            self.cdp_lmh = True
            self.V_local_lmh = vl
            self.lm_head = p(vl, self.H)
        elif tied:
            # the LM head keeps the replica's vocab shard; it is loaded from the embedding
            self.lm_head = p(self.V_local, self.H) if embed else self.embed
        if tied and (embed or lm_head) and self.lm_head is not self.embed:
            self.lm_head_from_embed = True

    def set_attention_dp(self):
        """Attention data parallelism on top of component DP (same replicas, same groups): the Q
        and O projections shard their heads over TP x DP ranks instead of the replica's TP
        ranks, so no replica holds a copy of another's Q / O weights.  Rank (replica d, TP
        position j) owns the ``Hq / (TP * DP)`` heads starting at ``j * Hq / TP + d * Hq /
        (TP * DP)``; together the DP column of TP position j owns that position's heads.  Per
        layer: all replicas' rows are gathered, each rank projects Q for its heads on all of
        them, an all-to-all over the DP column returns every replica its own rows with all the
        heads of its TP position; K / V (replica TP, as before) and attention run on the
        replica's own KV cache; the reverse all-to-all hands each rank all replicas' attention
        rows for its heads, its O shard makes partial sums that are all-reduced over TP x DP,
        and each replica keeps its rows.  With more KV heads than TP ranks (a whole number per
        TP x DP rank) K / V are sharded and exchanged with Q (Q+K+V variant), else they stay per
        replica (Q-only variant).  DP here is the attention-DP size k (k replicas).  Reference: attention DP, docs/design/parallelism/attention_dp.md,
        vllm_neuron/model/llama3/model.py:341-408,1125-1157."""
        if "attn" not in getattr(self, "cdp_groups", {}):
            raise ValueError("attention data parallelism needs its groups (set_component_dp)")
        W = self.cdp_groups["attn"][1].world
        if self.cfg.num_heads % W:
            raise ValueError(f"{self.cfg.num_heads} attention heads do not split over {W} ranks")
        self.cdp_attn = True
        self.Hq_w = self.cfg.num_heads // W
        # Q+K+V variant: with more KV heads than replica TP ranks, and a whole number of them per
        # TP x DP rank, K / V are sharded and exchanged like Q (no replica holds another's K / V
        # weights); otherwise K / V stay replica-TP (Q-only variant)
        nkv, t = self.cfg.num_kv_heads, self.tp.world
        self.Hkv_w = nkv // W if (nkv > t and nkv % W == 0) else 0
        p = lambda *s: torch.nn.Parameter(torch.empty(*s, dtype=self.dtype, device=self.device), requires_grad=False)
        for ly in self.layers:
            ly.q_w = p((self.Hq_w + 2 * self.Hkv_w) * self.D, self.H)
            ly.kv = None if self.Hkv_w else p(2 * self.Hkv * self.D, self.H)
            ly.o = p(self.H, self.Hq_w * self.D)
            del ly.qkv
            ly.qkv = None

    def _attention_dp(self, ly, x, res, b: ForwardBatch, T: int, k_cache, v_cache, kv_scale):
        """One attention block under attention data parallelism (see set_attention_dp); leaves
        ``x = post_norm(res += attention)`` for this replica's rows."""
        dc, cg = self.cdp_groups["attn"]
        D, Tm, Dh = dc.world, max(self.dp_tmax, T, 1), self.D
        hw = self.Hq_w * Dh
        kw = self.Hkv_w * Dh
        xall = self._gather_rows(x, T, Tm, dc)
        qw = L.gemm_out(xall, ly.q_w)                                     # [D * Tm, hw (+ 2 kw)]
        own = dc.all_to_all(qw.view(D, Tm, hw + 2 * kw).contiguous())  # [source d, Tm, .]
        own = own[:, :T]
        q_own = own[..., :hw].permute(1, 0, 2).reshape(T, D * hw)
        if self.Hkv_w:  # K and V heads of every source, in head order
            k_own = own[..., hw:hw + kw].permute(1, 0, 2).reshape(T, D * kw)
            v_own = own[..., hw + kw:].permute(1, 0, 2).reshape(T, D * kw)
            qkv = torch.cat([q_own, k_own, v_own], dim=1).contiguous()
        else:
            qkv = torch.cat([q_own, L.gemm_out(x[:T], ly.kv)], dim=1).contiguous()
        q = self.ws_q[:T]
        # (after the exchange the rows hold the replica TP position's heads in order: the
        # replica-TP qkv bias applies as is)
        ops.rope_kv_write(qkv, b.positions, self.cos_sin, self.Hq, self.Hkv, Dh, q, k_cache, v_cache,
                          b.slot_mapping, ly.q_norm, ly.k_norm, self.eps, rot_dim=self.cfg.rot_dim,
                          q_pos_scale=self.q_pos_scale, qkv_bias=self._f32(ly, "qkv_bias"),
                          positions3=b.positions3,
                          mrope_section=self.mrope_section, k_scale=kv_scale[0], v_scale=kv_scale[1])
        attn = self.ws_attn[:T]
        self._attention(q, attn, k_cache, v_cache, b, window=ly.window, sinks=ly.sinks, kv_scale=kv_scale)
        ap = attn.new_zeros(Tm, D, hw)
        ap[:T] = attn.view(T, D, hw)
        arecv = dc.all_to_all(ap.permute(1, 0, 2).contiguous())   # [source replica, Tm, hw]
        h = L.gemm_out(arecv.reshape(D * Tm, hw), ly.o)
        cg.all_reduce_(h)
        r = dc.rank
        own = h[r * Tm:r * Tm + T]
        if ly.o_bias is not None:
            own = own + ly.o_bias
        self._add_norm_rows(own, res, ly.post_norm, x, T)

    def _gather_rows(self, t: torch.Tensor, n: int, nmax: int, dc: GroupComm) -> torch.Tensor:
        """The DP column's replicas' first ``n`` rows of ``t`` (each padded to ``nmax``),
        replica-major."""
        D = dc.world
        tp_ = t.new_zeros((nmax,) + tuple(t.shape[1:]))
        tp_[:n] = t[:n]
        return dc.all_gather(tp_.unsqueeze(0).contiguous(), dim=0).reshape((D * nmax,) + tuple(t.shape[1:]))

    def _mlp_cdp(self, ly, x, res, nxt_norm, T: int):
        """Component-DP MLP: gather the replicas' rows, run this rank's MLP shard on all of
        them, all-reduce over every rank, keep this replica's rows."""
        dc, cg = self.cdp_groups["mlp"]
        Tm = max(self.dp_tmax, T, 1)
        xall = self._gather_rows(x, T, Tm, dc)
        if self.silu_blk:
            act = L.gemm_silu(xall, ly.gate_up)
        else:
            act = ops.silu_mul(L.gemm_out(xall, ly.gate_up))
        h = L.gemm_out(act, ly.down)
        cg.all_reduce_(h)
        r = dc.rank
        self._add_norm_rows(h[r * Tm:r * Tm + T], res, nxt_norm, x, T)

    def _embed_cdp(self, b: ForwardBatch, res: torch.Tensor, T: int):
        """Component-DP embedding: the replicas' token ids (device-resident ones resolved first)
        are gathered, looked up in this rank's vocab shard, all-reduced, own rows kept."""
        ids = b.input_ids[:T]
        if b.last_tok is not None:
            ids = torch.where(ids < 0, b.last_tok[(-ids - 1).clamp(min=0).long()].to(ids.dtype), ids)
        dc, cg = self.cdp_groups["embed"]
        Tm = max(self.dp_tmax, T, 1)
        iall = self._gather_rows(ids, T, Tm, dc)
        e = ops.embedding(iall, self.embed, self.vocab_start_emb, self.vocab_start_emb + self.V_local_emb)
        cg.all_reduce_(e)
        r = dc.rank
        res.copy_(e[r * Tm:r * Tm + T])

    def _logits_cdp(self, xs: torch.Tensor) -> torch.Tensor:
        """Component-DP LM head: gather the replicas' logits rows, this rank's vocab slice for
        all of them, all-gather the slices over every rank, keep this replica's rows."""
        S = xs.shape[0]
        dc, cg = self.cdp_groups["lm_head"]
        Sm = max(self.dp_smax, S, 1)
        xall = self._gather_rows(xs, S, Sm, dc)
        lg = L.gemm_out(xall, self.lm_head)
        lg = cg.all_gather(lg, dim=1)
        r = dc.rank
        return lg[r * Sm:r * Sm + S, :self.V]

    def _add_norm_rows(self, h, res, norm_w, x, T: int):
        """``res[:T] += h``, ``x[:T] = rmsnorm(res[:T])`` (h already reduced)."""
        ops.add_rmsnorm(h.contiguous(), res[:T], norm_w, self.eps, out=x[:T])

    def _allreduce_norm(self, acc, res, norm_w, x, fused: bool):
        """Decode-size row-parallel epilogue: ``res += all_reduce(acc)``, ``x = rmsnorm(res)``."""
        if fused:
            self.tp_fused.allreduce_norm(acc, res, norm_w, self.eps, x)
        else:
            self.tp.all_reduce_(acc)
            ops.add_rmsnorm(acc, res, norm_w, self.eps, out=x, clear_x=True)

    def _attention(self, q, attn, k_cache, v_cache, b: ForwardBatch, window: int = 0, sinks=None,
                   kv_scale: tuple[float, float] = (1.0, 1.0)):
        T = b.num_tokens
        ns = b.num_splits
        if self.dcp.world > 1:
            return self._attention_dcp(q, attn, k_cache, v_cache, b, kv_scale)
        part_o = part_l = None
        if ns > 1:
            part_o = self.ws_part_o[: ns * T * self.Hq * self.D].view(ns, T, self.Hq, self.D)
            part_l = self.ws_part_lse[: ns * T * self.Hq].view(ns, T, self.Hq)
        ops.paged_attention(q.view(T, self.Hq, self.D), k_cache, v_cache, b.block_tables, b.seq_lens,
                            b.q_start, b.work, b.decode, ns, self.scale, window=window, sinks=sinks,
                            out=attn.view(T, self.Hq, self.D), part_o=part_o, part_lse=part_l,
                            k_scale=kv_scale[0], v_scale=kv_scale[1], splits_dev=b.splits_dev,
                            prefill_rows=b.prefill_rows)

    def _attention_dcp(self, q, attn, k_cache, v_cache, b: ForwardBatch,
                       kv_scale: tuple[float, float]):
        """Decode context parallelism: this rank's cache holds one block-size slice of every
        ``dcp * block_size`` token window.  Q is all-gathered over the replica set (whose ranks
        share the KV heads), every rank attends over its own tokens and writes unmerged
        partials, one all-to-all hands each rank the partials of its own heads and the split
        merge kernel combines them by log-sum-exp (reference: all-gather Q, local attention,
        all-gather LSE, correction and reduce-scatter over heads,
        functional/attention/attention_decode.py:902-1062)."""
        d = self.dcp
        T, Hq, D, ns, W = b.num_tokens, self.Hq, self.D, b.num_splits, self.dcp.world
        qg = d.all_gather(q.view(T, Hq, D), dim=1)  # [T, W * Hq, D], heads in rank order
        po, pl = self._dcp_partials(ns, T, W * Hq, D, q.device)
        ops.paged_attention_partial(qg, k_cache, v_cache, b.block_tables, b.seq_lens_local,
                                    b.q_start, b.work, b.decode, ns, self.scale, po, pl,
                                    k_scale=kv_scale[0], v_scale=kv_scale[1],
                                    dcp_seq_lens=b.seq_lens, dcp_size=W, dcp_rank=d.rank)
        # chunk k of dim 0 (heads of rank k) goes to rank k; chunk k received comes from rank k
        ro = d.all_to_all(po.view(ns, T, W, Hq, D).permute(2, 0, 1, 3, 4).contiguous())
        rl = d.all_to_all(pl.view(ns, T, W, Hq).permute(2, 0, 1, 3).contiguous())
        ops.attn_combine(ro.view(W * ns, T, Hq, D), rl.view(W * ns, T, Hq),
                         out=attn.view(T, Hq, D))

    def _dcp_partials(self, ns: int, T: int, Hg: int, D: int, dev) -> tuple[torch.Tensor, torch.Tensor]:
        """Views ``[ns, T, Hg, D]`` / ``[ns, T, Hg]`` of one fp32 workspace kept on the model and
        grown (never shrunk) to the largest step seen: sized on the first decode step for the
        decode bound and on the first prefill chunk for the token budget, not allocated per
        layer."""
        n_o, n_l = ns * T * Hg * D, ns * T * Hg
        ws = getattr(self, "_dcp_ws", None)
        if ws is None or ws.numel() < n_o + n_l:
            cap = max(n_o + n_l, self.attn_splits_max * self.max_decode_tokens * Hg * (D + 1))
            self._dcp_ws = ws = torch.empty(cap, dtype=torch.float32, device=dev)
        return ws[:n_o].view(ns, T, Hg, D), ws[n_o:n_o + n_l].view(ns, T, Hg)

    def compute_logits(self, x: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        S = idx.shape[0]
        if S > self.ws_logits.shape[0]:  # draft verification rows beyond the preallocated ones
            xs = torch.empty(S, self.H, dtype=self.dtype, device=x.device)
            logits = torch.empty(S, self.V_local, dtype=self.dtype, device=x.device)
        else:
            xs = self.ws_logits_x[:S]
            logits = self.ws_logits[:S]
        torch.index_select(x, 0, idx, out=xs)
        if self.cdp_lmh:
            return self._logits_cdp(xs)
        if S <= L.SKINNY_MAX and x.is_cuda:
            L.gemm_skinny_bf16(xs, self.lm_head, out=logits)
        else:
            L.gemm_out(xs, self.lm_head, out=logits)
        if getattr(self, "skip_logits_gather", False):
            return logits  # vocab shard [S, V_local] (sampling data parallelism)
        if self.tp.world > 1:
            logits = self.tp.all_gather(logits, dim=1)
        return logits[:, : self.V]

    # ---------------------------------------------------------------- HF weight loading
    def load_hf_state_dict(self, get_tensor, names: set[str]):
        """Load from HF tensor names.  ``get_tensor(name)`` returns a CPU tensor."""
        from ..utils.weight_loader import load_dense_decoder

        load_dense_decoder(self, get_tensor, names)
