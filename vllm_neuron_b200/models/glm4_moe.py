"""GLM-4.5 / GLM-4.6 mixture-of-experts decoder (``Glm4MoeForCausalLM``) on the dense
attention path of :mod:`.llama`:

* attention: GQA with q/k/v bias, partial rotary embedding (``partial_rotary_factor``,
  neox pairs on the first ``rot_dim`` dims), optional q/k RMSNorm (``use_qk_norm``);
* the first ``first_k_dense_replace`` layers have a dense SwiGLU MLP, the others a MoE block:
  sigmoid router scores, experts ranked by ``score + e_score_correction_bias`` (the bias only
  selects), routing weights = the selected plain scores (optionally renormalised) times
  ``routed_scaling_factor``, plus an ungated shared expert of ``n_shared_experts`` times the
  expert width.

Group-limited routing (``n_group > 1`` with ``topk_group < n_group``) is not supported; the
GLM-4.5 family uses a single group.  The math follows the model's published definition (the
reference ports of the same family, and HF ``Glm4MoeForCausalLM``).
"""
from __future__ import annotations

import torch

from ..exceptions import UnsupportedConfigError
from ..ops import moe as M
from .llama import LlamaForCausalLM
from .qwen_moe import MoEMixin, load_moe_mlp


class Glm4MoeForCausalLM(MoEMixin, LlamaForCausalLM):
    route_mode = M.ROUTE_SIGMOID_BIAS_TOPK
    shared_gated = False

    def __init__(self, cfg, *args, **kw):
        raw = cfg.raw
        n_group, topk_group = raw.get("n_group") or 1, raw.get("topk_group") or 1
        if n_group > 1 and topk_group < n_group:
            raise UnsupportedConfigError("GLM MoE: group-limited routing (topk_group < n_group) is not supported")
        tp = kw.get("tp")
        W = tp.world if tp is not None else 1
        self.first_dense = int(raw.get("first_k_dense_replace", 1) or 0)
        self.routed_scale = float(raw.get("routed_scaling_factor", 1.0) or 1.0)
        self._init_moe(cfg, tp)
        n_shared = int(raw.get("n_shared_experts", 0) or 0)
        if (self.I_moe * n_shared) % W:
            raise UnsupportedConfigError("GLM MoE: shared expert width must split over the TP ranks")
        self.I_sh = self.I_moe * n_shared // W
        super().__init__(cfg, *args, **kw)
        self._post_init_moe()

    def _make_mlp(self, m, p, layer: int):
        m.is_moe = layer >= self.first_dense
        if m.is_moe:
            self._moe_params(m, p)
            m.router_bias = torch.nn.Parameter(torch.zeros(self.E, dtype=torch.float32, device=self.device),
                                               requires_grad=False)
        else:
            LlamaForCausalLM._make_mlp(self, m, p, layer)

    def _mlp(self, i, ly, x, res, nxt_norm, T, small, fused):
        if ly.is_moe:
            self._moe_mlp(ly, x, res, nxt_norm, T)
        else:
            LlamaForCausalLM._mlp(self, i, ly, x, res, nxt_norm, T, small, fused)

    def load_hf_state_dict(self, get_tensor, names: set[str]):
        from ..utils.weight_loader import load_dense_decoder, load_dense_mlp

        def mlp_loader(model, ly, get, nm, p):
            if ly.is_moe:
                load_moe_mlp(model, ly, get, nm, p)
            else:
                load_dense_mlp(model, ly, get, p)

        load_dense_decoder(self, get_tensor, names, mlp_loader=mlp_loader)
