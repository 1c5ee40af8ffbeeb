"""Hybrid linear-attention MoE decoder of the Qwen3.5 / Qwen3.6 family (text part), e.g.
``Qwen3_5MoeForCausalLM``: a repeating pattern of gated DeltaNet layers and gated full-attention
layers, each followed by a routed-experts MLP with a sigmoid-gated shared expert.

Per layer (TP world W; heads and channels are split over the ranks):

  linear attention (gated DeltaNet)
    p   = x @ W_in^T                          one GEMM for q|k|v, z, b, a
    c   = silu(causal_conv1d(p[q|k|v]))        conv window kept in the state cache
    o   = gated_delta_rule(c, z, a, b)         recurrent state S [dk, dv] per value head in the
                                               state cache; gated RMSNorm with silu(z) fused
    h   = o @ W_out^T -> all-reduce
  gated full attention
    p   = x @ W_qkvg^T                         q | k | v | output gate
    q,k = rope(rmsnorm(q), rmsnorm(k)), k/v -> paged KV cache
    a   = paged_attention(q) * sigmoid(gate)
    h   = a @ W_o^T -> all-reduce
  x = rmsnorm(residual += h); MoE MLP (+ shared expert); x = rmsnorm(residual += mlp)

RMSNorm weights of this family are stored as offsets from 1 (``(1 + w) * x``); they are
converted to plain scales when loaded.  Only the full-attention layers have a paged KV
cache; the linear layers keep per-request state (conv window + recurrent state) in a cache
indexed by the request's slot.  The reference has no linear-attention model; the math
follows the HF implementation and the published gated delta rule (Yang et al., 2024).
"""
from __future__ import annotations

import torch

from .. import ops
from ..ops import deltanet as DN
from ..ops import linear as L
from .llama import ForwardBatch
from .qwen_moe import MoEMixin, Qwen3MoeForCausalLM


def num_state_slots(max_seqs: int) -> int:
    """State-cache slots: the runner's request slots (2 * max_num_seqs + 8, the last is padding)."""
    return 2 * max_seqs + 8


class Qwen3_5MoeForCausalLM(Qwen3MoeForCausalLM):
    component_dp_parts = ("embed", "lm_head")  # gated attention / DeltaNet stay per replica
    supports_dcp = False  # sinks / sliding windows / linear-attention state
    supports_prefix_caching = False

    # "auto" (chunked WY form for steps with a full 64-token chunk, else token by token),
    # "chunked" or "recurrent"
    deltanet_mode = "auto"

    def __init__(self, cfg, *args, **kw):
        tp = kw.get("tp")
        W = tp.world if tp is not None else 1
        self.lin_Hk = cfg.linear_num_key_heads // W
        self.lin_Hv = cfg.linear_num_value_heads // W
        self.lin_dk = cfg.linear_key_head_dim
        self.lin_dv = cfg.linear_value_head_dim
        self.conv_K = cfg.linear_conv_kernel_dim
        self.conv_dim = 2 * self.lin_Hk * self.lin_dk + self.lin_Hv * self.lin_dv
        self.lin_proj = self.conv_dim + self.lin_Hv * self.lin_dv + 2 * self.lin_Hv
        self.is_linear = [cfg.layer_is_linear(i) for i in range(cfg.num_layers)]
        self.attn_layers = [i for i in range(cfg.num_layers) if not self.is_linear[i]]
        self.kv_index = {l: j for j, l in enumerate(self.attn_layers)}
        self.lin_index = {l: j for j, l in enumerate(i for i in range(cfg.num_layers) if self.is_linear[i])}
        super().__init__(cfg, *args, **kw)
        max_seqs = kw.get("max_seqs", 256)
        S = num_state_slots(max_seqs)
        nl = len(self.lin_index)
        self.conv_state = torch.zeros(nl, S, self.conv_dim, self.conv_K - 1, dtype=self.dtype, device=self.device)
        self.ssm_state = torch.zeros(nl, S, self.lin_Hv, self.lin_dk, self.lin_dv, dtype=torch.float32,
                                     device=self.device)
        T = self.max_tokens
        self.ws_lin_proj = torch.zeros(T, self.lin_proj, dtype=self.dtype, device=self.device)
        self.ws_lin_conv = torch.zeros(T, self.conv_dim, dtype=self.dtype, device=self.device)
        self.ws_lin_out = torch.zeros(T, self.lin_Hv * self.lin_dv, dtype=self.dtype, device=self.device)
        self.ws_qkvg = torch.zeros(T, self.qkv_out + self.Hq * self.D, dtype=self.dtype, device=self.device)

    # ------------------------------------------------------------------ parameters
    def _make_attn(self, m, p, layer: int):
        if self.is_linear[layer]:
            m.w_in = p(self.lin_proj, self.H)
            m.conv_w = p(self.conv_dim, self.conv_K)
            m.A_log = torch.nn.Parameter(torch.zeros(self.lin_Hv, dtype=torch.float32, device=self.device),
                                         requires_grad=False)
            m.dt_bias = torch.nn.Parameter(torch.ones(self.lin_Hv, dtype=torch.float32, device=self.device),
                                           requires_grad=False)
            m.gnorm_w = p(self.lin_dv)
            m.out_proj = p(self.H, self.lin_Hv * self.lin_dv)
        else:
            m.qkvg = p(self.qkv_out + self.Hq * self.D, self.H)
            m.q_norm = p(self.D)
            m.k_norm = p(self.D)
            m.o = p(self.H, self.Hq * self.D)

    @property
    def num_kv_layers(self) -> int:
        return len(self.attn_layers)


    @torch.no_grad()
    def init_random(self, seed: int = 0, std: float = 0.02):
        super().init_random(seed, std)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 1000 + 11 + self.tp.rank)
        for i, ly in enumerate(self.layers):
            if self.is_linear[i]:
                ly.A_log.copy_(torch.empty(self.lin_Hv, device=self.device).uniform_(1, 16, generator=g).log())
                ly.dt_bias.fill_(1.0)
                ly.gnorm_w.fill_(1.0)
                ly.conv_w.normal_(0.0, 0.3, generator=g)

    def load_hf_state_dict(self, get_tensor, names: set[str]):
        from ..utils.weight_loader import load_qwen3_5

        load_qwen3_5(self, get_tensor, names)

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, b: ForwardBatch) -> torch.Tensor:
        T = b.num_tokens
        tp = self.tp
        res = self.ws_residual[:T]
        x = self.ws_x[:T]
        if self.cdp_embed:
            self._embed_cdp(b, res, T)
        else:
            ops.embedding(b.input_ids, self.embed, self.vocab_start, self.vocab_start + self.V_local, out=res,
                          last_tok=b.last_tok)
            tp.all_reduce_(res)
        ops.rmsnorm(res, self.layers[0].input_norm, self.eps, out=x)
        cs = self.capture
        if cs is not None and cs.point("model.embed_tokens", res):
            ops.rmsnorm(res, self.layers[0].input_norm, self.eps, out=x)
        nL = len(self.layers)
        slots = b.seq_slots
        for i, ly in enumerate(self.layers):
            h = self.ws_h[:T]
            if self.is_linear[i]:
                li = self.lin_index[i]
                proj = _linear(x, ly.w_in, self.ws_lin_proj[:T])
                cd, Vd, Hv = self.conv_dim, self.lin_Hv * self.lin_dv, self.lin_Hv
                conv = DN.causal_conv1d(proj[:, :cd], ly.conv_w, b.q_start, b.seq_lens, slots,
                                        self.conv_state[li], self.ws_lin_conv[:T])
                z = proj[:, cd:cd + Vd]
                bb = proj[:, cd + Vd:cd + Vd + Hv]
                aa = proj[:, cd + Vd + Hv:cd + Vd + 2 * Hv]
                core = DN.gated_delta_rule(conv, z, aa, bb, ly.A_log, ly.dt_bias, ly.gnorm_w, self.eps,
                                           b.q_start, b.seq_lens, slots, self.ssm_state[li],
                                           self.ws_lin_out[:T], self.lin_Hk, self.lin_Hv,
                                           mode=DN.pick_mode(T, b.max_q_len, self.deltanet_mode))
                _linear(core, ly.out_proj, h)
            else:
                k_cache, v_cache = self.kv_caches[self.kv_index[i]]
                ks, vs = self.kv_scale(self.kv_index[i])
                qkvg = _linear(x, ly.qkvg, self.ws_qkvg[:T])
                q = self.ws_q[:T]
                ops.rope_kv_write(qkvg[:, :self.qkv_out], b.positions, self.cos_sin, self.Hq, self.Hkv, self.D,
                                  q, k_cache, v_cache, b.slot_mapping, ly.q_norm, ly.k_norm, self.eps,
                                  rot_dim=self.cfg.rot_dim, k_scale=ks, v_scale=vs)
                attn = self.ws_attn[:T]
                self._attention(q, attn, k_cache, v_cache, b, kv_scale=(ks, vs))
                DN.sigmoid_gate_mul(attn, qkvg[:, self.qkv_out:])
                _linear(attn, ly.o, h)
            tp.all_reduce_(h)
            ops.add_rmsnorm(h, res, ly.post_norm, self.eps, out=x)
            nxt_norm = self.layers[i + 1].input_norm if i + 1 < nL else self.final_norm
            self._moe_mlp(ly, x, res, nxt_norm, T)
            if cs is not None and cs.point(f"model.layers.{i}", res):
                ops.rmsnorm(res, nxt_norm, self.eps, out=x)
        if cs is not None:
            cs.point("model.norm", x)
        if b.want_hidden:
            return x.index_select(0, b.logits_indices.long())
        logits = self.compute_logits(x, b.logits_indices)
        if cs is not None:
            cs.point("lm_head", logits, logits=True)
        return logits


def _linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """bf16 ``out = x @ w^T`` on the tcgen05 GEMM (skinny variant for decode batches)."""
    if x.is_cuda and x.shape[0] <= L.SKINNY_MAX:
        return L.gemm_skinny_bf16(x, w, out=out)
    return L.gemm_out(x, w, out=out)
