"""Qwen mixture-of-experts decoders on the dense attention path of :mod:`.llama`:

* ``Qwen3MoeForCausalLM``: softmax routing over all experts, top-k, optional renormalisation
  (``norm_topk_prob``), SiLU experts, QK-norm attention;
* ``Qwen2MoeForCausalLM``: the same plus a shared expert whose output is scaled by
  ``sigmoid(x . shared_expert_gate)``.

Experts are sharded by index over the tensor-parallel ranks (expert parallelism over the TP
group); the shared expert is sharded by its intermediate dimension like a dense MLP, so the
partial outputs of all ranks sum to the full block output in the all-reduce.  The shared
expert's gate is appended to the router as row ``E`` (one GEMM for both).

Reference: the MoE block semantics of vllm_neuron/functional/moe/moe_block_tkg.py:306
(router + experts + shared expert) and router.py:72 (softmax -> top-k -> renormalise).
"""
from __future__ import annotations

import torch

from .. import ops
from ..ops import moe as M
from .llama import LlamaForCausalLM


class MoEMixin:
    """Routed-experts MLP for decoder models built on :class:`LlamaForCausalLM`."""

    route_mode = M.ROUTE_SOFTMAX_TOPK
    expert_act = M.ACT_SILU
    shared_gated = True   # shared expert scaled by sigmoid(x . gate) (router row E)
    routed_scale = 1.0    # multiplies the routing weights

    def _init_moe(self, cfg, tp):
        W = tp.world if tp is not None else 1
        self.E = cfg.num_experts
        self.topk = cfg.num_experts_per_tok
        self._shard_experts(W)
        self.I_moe = cfg.moe_intermediate_size or cfg.intermediate_size
        self.I_sh = (cfg.shared_expert_intermediate_size or 0) // W
        self.renorm = bool(cfg.norm_topk_prob)

    def _shard_experts(self, W: int):
        """Experts by index over the TP group (partials summed by the all-reduce), or over the
        EP group with all-to-all token exchange when wide EP is configured."""
        from ..parallel import state as ps

        self.a2a = None
        st = ps.get_parallel_state()
        if getattr(st, "ep_all2all", False) and st.ep.world > 1:
            # wide EP: experts sharded over the EP group, whose ranks hold different tokens
            # (data-parallel replicas); tokens travel by all-to-all (parallel/all2all.py)
            if W > 1:
                raise NotImplementedError("all-to-all expert parallelism needs TP=1 per data-parallel replica")
            from ..parallel.all2all import All2AllManager

            self.a2a = All2AllManager(st.ep.group, st.ep.rank, st.ep.world, self.E)
            self.e_local = self.a2a.e_local
            self.supports_cuda_graphs = False  # host-side split sizes per exchange
        else:
            assert self.E % W == 0, f"{self.E} experts not divisible by TP={W}"
            self.e_local = self.E // W

    def _post_init_moe(self):
        self.e_start = self.a2a.e_start if self.a2a is not None else self.tp.rank * self.e_local
        self.moe_ws = None
        self.ep_fused = None
        if self.device.type == "cuda":
            self.moe_ws = M.MoEWorkspace.create(self.max_tokens + self.tp.world, self.topk, self.E, self.e_local, self.H,
                                                self.I_moe, self.device, shared_inter=self.I_sh)
            from .. import envs

            if self.a2a is not None and not envs.VLLM_B200_DISABLE_FUSED_COMM:
                # wide EP on the GPU: the device-side exchange over NVLink peer memory
                from ..parallel import state as ps
                from ..parallel.ep_fused import EPFusedExchange

                st = ps.get_parallel_state()
                cap = self.max_tokens + self.tp.world
                self.ep_fused = EPFusedExchange(st.ep.group, st.ep.rank, st.ep.world, self.E, self.topk,
                                                self.H, cap, self.device, st.cpu)
                R = self.ep_fused.rows_cap
                self.ep_ws = M.MoEWorkspace.create(R, self.topk, self.E, self.e_local, self.H, self.I_moe,
                                                   self.device)
                self.ep_y = torch.zeros(R, self.H, dtype=torch.bfloat16, device=self.device)
                self.ep_out = torch.zeros(cap, self.H, dtype=torch.bfloat16, device=self.device)

    def _moe_params(self, m, p):
        m.router = p(self.E + (1 if self.I_sh and self.shared_gated else 0), self.H)
        m.w_gu = p(self.e_local, 2 * self.I_moe, self.H)
        m.w_down = p(self.e_local, self.H, self.I_moe)
        if self.I_sh:
            m.sh_gu = p(2 * self.I_sh, self.H)
            m.sh_down = p(self.H, self.I_sh)
        else:
            m.sh_gu = m.sh_down = None

    def _moe_mlp(self, ly, x, res, nxt_norm, T):
        h = self.ws_h[:T]
        if self.a2a is not None:
            self._moe_all2all(ly, x[:T], h)
        else:
            M.moe_block(x, ly.router, ly.w_gu, ly.w_down, self.topk, self.route_mode, self.renorm,
                        router_b=getattr(ly, "router_bias", None), act=self.expert_act,
                        e_start=self.e_start, ws=self.moe_ws, out=h, num_experts=self.E,
                        shared_gu=ly.sh_gu, shared_down=ly.sh_down, routed_scale=self.routed_scale,
                        shared_gated=self.shared_gated)
        self._reduce_norm(h, res, nxt_norm, x)

    def _moe_all2all(self, ly, x, out, b_gu=None, b_down=None, alpha=1.702, limit=7.0):
        """Route the local tokens, dispatch them to the ranks owning their experts, run this
        rank's experts on the rows received, send the pre-reduced rows back and sum them per
        token; the shared expert (replicated) runs on the local tokens.  Reference:
        vllm_neuron/parallel/all2all.py:33-641 with functional/moe/moe_tkg.py:17 on the A2A-v
        input layout."""
        from ..ops import ep as EP
        from ..ops import linear as L

        E = self.E
        if x.is_cuda:
            logits = L.gemm_out(x, ly.router)
        else:
            logits = (x.float() @ ly.router.float().t()).to(x.dtype)
        sh_gu = getattr(ly, "sh_gu", None)
        gated = sh_gu is not None and self.shared_gated
        ids, w = M.route(logits, self.topk, self.route_mode, self.renorm, getattr(ly, "router_bias", None),
                         num_experts=E, scale=self.routed_scale)
        if x.is_cuda and self.ep_fused is not None:
            # device-side exchange: rows land in this rank's receive buffer, the experts run on
            # its static row bound, reduced rows go back into the owners' combine slots
            ex = self.ep_fused
            ex.dispatch(x, ids, w)
            rows, rids, rw = ex.recv()
            M._experts_cuda(rows, rids, rw, ly.w_gu, ly.w_down, self.topk, b_gu, b_down, self.expert_act,
                            alpha, limit, self.e_start, self.ep_ws, self.ep_y, None, None, None, None, 0)
            ex.ret(self.ep_y)
            y = ex.combine(self.ep_out[:x.shape[0]]).float()
        else:
            plan, rows, aff = self.a2a.dispatch(x, ids, w)
            lids, lw = EP.local_routing(aff, self.e_start, self.topk)
            part = M.moe_experts(rows, lids, lw, ly.w_gu, ly.w_down, b_gu, b_down, self.expert_act, alpha,
                                 limit, e_start=self.e_start)
            y = self.a2a.combine(part, plan).float()
        if sh_gu is not None:
            if x.is_cuda:
                from ..ops.activation import silu_mul

                sh = L.gemm_out(silu_mul(L.gemm_out(x, ly.sh_gu)), ly.sh_down).float()
            else:
                sh = M.shared_expert_ref(x, ly.sh_gu, ly.sh_down)
            gate = torch.sigmoid(logits[:, E:E + 1].float()) if gated else 1.0
            y = y + gate * sh
        out.copy_(y.to(out.dtype))


class Qwen3MoeForCausalLM(MoEMixin, LlamaForCausalLM):
    def __init__(self, cfg, *args, **kw):
        self._init_moe(cfg, kw.get("tp"))
        super().__init__(cfg, *args, **kw)
        self._post_init_moe()

    def _make_mlp(self, m, p, layer: int):
        self._moe_params(m, p)

    def _mlp(self, i, ly, x, res, nxt_norm, T, small, fused):
        self._moe_mlp(ly, x, res, nxt_norm, T)

    def load_hf_state_dict(self, get_tensor, names: set[str]):
        from ..utils.weight_loader import load_dense_decoder

        load_dense_decoder(self, get_tensor, names, mlp_loader=load_moe_mlp)


class Qwen2MoeForCausalLM(Qwen3MoeForCausalLM):
    pass


@torch.no_grad()
def load_moe_mlp(model, ly, get_tensor, names: set[str], p: str):
    """Router (+ shared expert gate), experts ``[e_start, e_start + e_local)`` and the TP shard
    of the shared expert, from fused (``experts.gate_up_proj [E, 2I, H]``) or per-expert
    (``experts.{e}.gate_proj.weight``) checkpoints."""
    from ..utils.weight_loader import _copy, shard_cols, shard_rows

    W, r = model.tp.world, model.tp.rank
    e0, el = model.e_start, model.e_local
    router = get_tensor(p + "mlp.gate.weight")
    if model.I_sh and model.shared_gated:
        router = torch.cat([router, get_tensor(p + "mlp.shared_expert_gate.weight").reshape(1, -1)], 0)
    _copy(ly.router, router, p + "router")
    if getattr(ly, "router_bias", None) is not None:  # selection-only correction bias (GLM-4.5)
        _copy(ly.router_bias, get_tensor(p + "mlp.gate.e_score_correction_bias").float(), p + "router_bias")
    fused = p + "mlp.experts.gate_up_proj"
    if fused in names:
        gu = get_tensor(fused)[e0:e0 + el]
        dn = get_tensor(p + "mlp.experts.down_proj")[e0:e0 + el]
    else:
        gu = torch.stack([torch.cat([get_tensor(f"{p}mlp.experts.{e}.gate_proj.weight"),
                                     get_tensor(f"{p}mlp.experts.{e}.up_proj.weight")], 0)
                          for e in range(e0, e0 + el)])
        dn = torch.stack([get_tensor(f"{p}mlp.experts.{e}.down_proj.weight") for e in range(e0, e0 + el)])
    _copy(ly.w_gu, gu, p + "w_gu")
    _copy(ly.w_down, dn, p + "w_down")
    if model.I_sh:
        sp = p + ("mlp.shared_experts." if p + "mlp.shared_experts.gate_proj.weight" in names
                  else "mlp.shared_expert.")
        g = shard_rows(get_tensor(sp + "gate_proj.weight"), W, r)
        u = shard_rows(get_tensor(sp + "up_proj.weight"), W, r)
        _copy(ly.sh_gu, torch.cat([g, u], 0), sp + "gate_up")
        _copy(ly.sh_down, shard_cols(get_tensor(sp + "down_proj.weight"), W, r), sp + "down")
