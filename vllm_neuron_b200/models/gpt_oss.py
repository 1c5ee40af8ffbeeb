"""GPT-OSS (``GptOssForCausalLM``): alternating sliding-window (128) / full attention with learned
per-head sinks, QKV and output biases, YaRN RoPE, and a mixture-of-experts MLP (top-k softmax
routing with a router bias, clamped SwiGLU with alpha, per-expert biases).

Attention runs on the dense decoder path of :mod:`.llama` (the paged attention kernel takes
the layer's window and sinks).  The MLP is :func:`vllm_neuron_b200.ops.moe.moe_block`.  Experts
are sharded across the tensor-parallel ranks (expert parallelism over the TP group): rank r
holds experts ``[r * E/W, (r + 1) * E/W)``, computes their contribution for every token and
the partial outputs are summed by the all-reduce that also serves attention-TP.

MXFP4 checkpoints (``*_blocks`` uint8 nibbles + ``*_scales`` e8m0 per 32 elements) are
dequantized to bf16 when loaded (:func:`dequant_mxfp4`).

Reference: vllm_neuron/model/gpt_oss/model_bf16.py (attention with sinks :393,721,770,938,
YaRN :142-232, MoE :982-1443), model_mxfp4.py and weight_loaders_mxfp4.py.
"""
from __future__ import annotations

import torch

from .. import envs, ops
from ..ops import linear as L
from ..ops import moe as M
from .llama import LlamaForCausalLM
from .qwen_moe import MoEMixin

# e2m1 code points (sign bit 3, exponent bits 2-1, mantissa bit 0)
_FP4_VALUES = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


def dequant_mxfp4(blocks: torch.Tensor, scales: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """``blocks [..., G, 16]`` uint8 (two e2m1 values per byte, low nibble first) and
    ``scales [..., G]`` uint8 (e8m0, bias 127) -> ``[..., G * 32]``."""
    lut = torch.tensor(_FP4_VALUES, dtype=torch.float32, device=blocks.device)
    b = blocks.to(torch.int64)
    lo = lut[b & 0x0F]
    hi = lut[b >> 4]
    v = torch.stack([lo, hi], dim=-1).reshape(*blocks.shape[:-1], 32)
    e = scales.to(torch.int32) - 127
    v = v * torch.pow(torch.tensor(2.0, device=blocks.device), e.to(torch.float32))[..., None]
    return v.reshape(*blocks.shape[:-2], blocks.shape[-2] * 32).to(dtype)


def quant_mxfp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Round ``w [..., K]`` (K % 32 == 0) to MXFP4: returns ``(blocks [..., K/32, 16], scales)``.
    Used to build random MXFP4 experts with the checkpoint format."""
    lut = torch.tensor(_FP4_VALUES[:8], dtype=torch.float32, device=w.device)
    x = w.float().reshape(*w.shape[:-1], w.shape[-1] // 32, 32)
    amax = x.abs().amax(-1).clamp_min(1e-30)
    e = torch.clamp(torch.ceil(torch.log2(amax / 6.0)), -127, 127)
    scaled = x / torch.pow(torch.tensor(2.0, device=w.device), e)[..., None]
    mag = scaled.abs().clamp(max=6.0)
    idx = (mag[..., None] - lut).abs().argmin(-1)
    code = idx | ((scaled < 0).to(torch.int64) << 3)
    code = code.reshape(*code.shape[:-1], 16, 2)
    blocks = (code[..., 0] | (code[..., 1] << 4)).to(torch.uint8)
    return blocks, (e + 127).to(torch.uint8)


def _quant_experts(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """MXFP4-quantize ``w [E, N, K]`` expert by expert (bounded temporary memory)."""
    bl, sc = [], []
    for e in range(w.shape[0]):
        b, s = quant_mxfp4(w[e])
        bl.append(b)
        sc.append(s)
    return torch.stack(bl), torch.stack(sc)


class GptOssForCausalLM(MoEMixin, LlamaForCausalLM):
    supports_dcp = False  # sinks / sliding windows / linear-attention state
    route_mode = M.ROUTE_TOPK_SOFTMAX
    expert_act = M.ACT_GPTOSS
    renorm = True

    def __init__(self, cfg, *args, **kw):
        W = kw.get("tp").world if kw.get("tp") is not None else 1
        self.E = cfg.num_experts
        self.topk = cfg.num_experts_per_tok
        self._shard_experts(W)  # by index over TP, or over the EP group with all-to-all
        self.I_moe = cfg.intermediate_size
        super().__init__(cfg, *args, **kw)
        self.e_start = self.a2a.e_start if self.a2a is not None else self.tp.rank * self.e_local
        p = lambda *s: torch.nn.Parameter(torch.empty(*s, dtype=self.dtype, device=self.device),
                                          requires_grad=False)
        for ly in self.layers:
            ly.o_bias = p(self.H)
            ly.sinks = torch.nn.Parameter(torch.zeros(self.Hq, dtype=torch.float32, device=self.device),
                                          requires_grad=False)
        self.moe_ws = None
        if self.device.type == "cuda":
            self.moe_ws = M.MoEWorkspace.create(self.max_tokens + self.tp.world, self.topk, self.E, self.e_local, self.H,
                                                self.I_moe, self.device)
        # MXFP4 copies of the experts for decode-sized batches (K = H for gate/up, I for down
        # must be multiples of 64); the bf16 copies serve prefill.
        self.use_fp4 = self.device.type == "cuda" and self.H % 64 == 0 and self.I_moe % 64 == 0
        self.fp4_max_tokens = envs.VLLM_B200_FP4_DECODE_MAX_TOKENS
        for ly in self.layers:
            ly.fp4_gu = ly.fp4_down = None

    def _make_mlp(self, m, p, layer: int):
        m.router = p(self.E, self.H)
        m.router_bias = torch.nn.Parameter(torch.zeros(self.E, dtype=torch.float32, device=self.device),
                                           requires_grad=False)
        m.w_gu = p(self.e_local, 2 * self.I_moe, self.H)
        m.b_gu = p(self.e_local, 2 * self.I_moe)
        m.w_down = p(self.e_local, self.H, self.I_moe)
        m.b_down = p(self.e_local, self.H)

    @torch.no_grad()
    def set_expert_mxfp4(self, ly, gu_blocks=None, gu_scales=None, dn_blocks=None, dn_scales=None):
        """Install the layer's MXFP4 experts: from checkpoint blocks/scales (gate/up rows in
        this model's gate-then-up order), or by quantizing the current bf16 weights.  The expert
        stacks become :class:`~..ops.linear.MXFP4Weight` (the bf16 copies are dropped): every
        batch runs them W4A16 on the tcgen05 grouped GEMM, and decode batches of at most
        ``VLLM_B200_FP4_DECODE_MAX_TOKENS`` tokens may use the fp4 mma.sync kernel on its own
        packed tiles instead (0 disables it)."""
        if not self.use_fp4:
            return
        if gu_blocks is None:
            if isinstance(ly.w_gu, L.MXFP4Weight):
                return
            gu_blocks, gu_scales = _quant_experts(ly.w_gu)
            dn_blocks, dn_scales = _quant_experts(ly.w_down)
        dev = self.device
        gu = L.MXFP4Weight.from_blocks(gu_blocks.to(dev), gu_scales.to(dev))
        dn = L.MXFP4Weight.from_blocks(dn_blocks.to(dev), dn_scales.to(dev))
        if self.fp4_max_tokens > 0:
            ly.fp4_gu = M.pack_mxfp4(gu_blocks.to(dev), gu_scales.to(dev))
            ly.fp4_down = M.pack_mxfp4(dn_blocks.to(dev), dn_scales.to(dev))
        for name, w in (("w_gu", gu), ("w_down", dn)):
            if name in ly._parameters:
                del ly._parameters[name]
            setattr(ly, name, w)
        if dev.type == "cuda":
            torch.cuda.empty_cache()

    @torch.no_grad()
    def quantize_mxfp8(self) -> int:
        """MXFP8 experts on the block-scaled tensor cores: each MXFP4 expert stack is re-encoded
        losslessly as MXFP8 (e2m1 values are e4m3 values, the e8m0 scales carry over), zero-padded
        to K in 128s and 128-row experts (hidden 2880 -> 2944), and served W8A8 by the grouped
        GEMM with the expert-sorted activations quantized to MXFP8; the fp4 decode copies are
        dropped.  Dense projections whose K is a multiple of 128 become MXFP8 as well."""
        n = super().quantize_mxfp8()
        rup = lambda v: -(-v // 128) * 128
        for ly in self.layers:
            if not isinstance(ly.w_gu, L.MXFP4Weight):
                continue
            gu = L.MXFP8Weight.from_mxfp4(ly.w_gu, k_pad=rup(self.H))
            dn = L.MXFP8Weight.from_mxfp4(ly.w_down, k_pad=rup(self.I_moe), n_pad=rup(self.H))
            ly.w_gu, ly.w_down = gu, dn
            ly.fp4_gu = ly.fp4_down = None
            n += 2
        self.mx_linears = n
        if self.device.type == "cuda":
            torch.cuda.empty_cache()
        return n

    def _mlp(self, i, ly, x, res, nxt_norm, T, small, fused):
        h = self.ws_h[:T]
        if self.a2a is not None:
            self._moe_all2all(ly, x[:T], h, b_gu=ly.b_gu, b_down=ly.b_down, alpha=self.cfg.swiglu_alpha,
                              limit=self.cfg.swiglu_limit)
            self._reduce_norm(h, res, nxt_norm, x)
            return
        M.moe_block(x, ly.router, ly.w_gu, ly.w_down, self.topk, M.ROUTE_TOPK_SOFTMAX,
                    router_b=ly.router_bias, b_gu=ly.b_gu,
                    b_down=ly.b_down,  # each assignment is computed on exactly one rank
                    act=M.ACT_GPTOSS, alpha=self.cfg.swiglu_alpha, limit=self.cfg.swiglu_limit,
                    e_start=self.e_start, ws=self.moe_ws, out=h, fp4_gu=ly.fp4_gu,
                    fp4_down=ly.fp4_down, fp4_max_tokens=self.fp4_max_tokens)
        self._reduce_norm(h, res, nxt_norm, x)

    @torch.no_grad()
    def init_random(self, seed: int = 0, std: float = 0.02):
        super().init_random(seed, std)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 1000 + 7 + self.tp.rank)
        for ly in self.layers:
            ly.sinks.normal_(0.0, 1.0, generator=g)
            self.set_expert_mxfp4(ly)

    def load_hf_state_dict(self, get_tensor, names: set[str]):
        from ..utils.weight_loader import load_gpt_oss

        load_gpt_oss(self, get_tensor, names)
