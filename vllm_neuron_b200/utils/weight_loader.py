"""HF checkpoint -> sharded, fused device parameters.

Transforms (per TP rank ``r`` of ``W``):
  * q/k/v projections are sliced by heads and concatenated into one ``qkv`` matrix; KV heads
    are replicated when ``W > num_kv_heads`` (rank r uses KV head ``r // (W / Hkv)``);
  * gate/up are sliced by rows and interleaved in 128-row blocks for the SwiGLU epilogue;
  * o_proj / down_proj are sliced by input columns (row-parallel);
  * embedding / LM head are sliced by vocabulary rows (last shard zero-padded).

Reference: vllm_neuron/utils/weight_loader.py:15-917 (sharding_weight_loader,
fused_qkv_weight_loader with KV replication, padding loaders).
"""
from __future__ import annotations

import collections

from typing import Callable

import torch

from ..ops import linear as L


def shard_rows(t: torch.Tensor, world: int, rank: int, pad_to: int | None = None) -> torch.Tensor:
    n = t.shape[0]
    per = pad_to if pad_to is not None else n // world
    s = t[rank * per: min((rank + 1) * per, n)]
    if s.shape[0] < per:
        s = torch.cat([s, torch.zeros((per - s.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype)], 0)
    return s


def shard_cols(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    per = t.shape[1] // world
    return t[:, rank * per:(rank + 1) * per]


def fused_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, num_heads: int, num_kv: int,
              head_dim: int, world: int, rank: int) -> torch.Tensor:
    hq = num_heads // world
    qs = q.view(num_heads, head_dim, -1)[rank * hq:(rank + 1) * hq].reshape(hq * head_dim, -1)
    if world >= num_kv:
        kv_idx = rank // (world // num_kv)
        ks = k.view(num_kv, head_dim, -1)[kv_idx:kv_idx + 1].reshape(head_dim, -1)
        vs = v.view(num_kv, head_dim, -1)[kv_idx:kv_idx + 1].reshape(head_dim, -1)
    else:
        hk = num_kv // world
        ks = k.view(num_kv, head_dim, -1)[rank * hk:(rank + 1) * hk].reshape(hk * head_dim, -1)
        vs = v.view(num_kv, head_dim, -1)[rank * hk:(rank + 1) * hk].reshape(hk * head_dim, -1)
    return torch.cat([qs, ks, vs], 0)


def _copy(dst: torch.nn.Parameter, src: torch.Tensor, name: str):
    if tuple(dst.shape) != tuple(src.shape):
        raise ValueError(f"{name}: shape {tuple(src.shape)} does not match parameter {tuple(dst.shape)}")
    dst.data.copy_(src.to(dst.dtype))


@torch.no_grad()
def _vocab_shards(model, W: int, r: int):
    """(world, rank, rows) of the embedding and of the LM head: over the component group under
    component data parallelism, else over TP."""
    grp = getattr(model, "cdp_groups", {})
    eg, hg = grp.get("embed", (None, None))[1], grp.get("lm_head", (None, None))[1]
    e = (eg.world, eg.rank, model.V_local_emb) if getattr(model, "cdp_embed", False) else (W, r, model.V_local)
    h = (hg.world, hg.rank, model.V_local_lmh) if getattr(model, "cdp_lmh", False) else (W, r, model.V_local)
    return e, h


def _load_attention_dp(model, ly, q, k, v, o, W: int, r: int, p: str):
    """Attention data parallelism: Q / O heads of this (replica, TP position) sub-group; K / V
    of the sub-group (Q+K+V variant) or of the replica's TP position (Q-only variant)."""
    cfg = model.cfg
    hq_w, hk_w, dh = model.Hq_w, model.Hkv_w, cfg.head_dim
    d = model.cdp_groups["attn"][0].rank
    h0 = r * (cfg.num_heads // W) + d * hq_w
    qs = q[h0 * dh:(h0 + hq_w) * dh]
    if hk_w:  # this rank's K / V heads follow its Q heads
        k0 = r * (cfg.num_kv_heads // W) + d * hk_w
        qs = torch.cat([qs, k[k0 * dh:(k0 + hk_w) * dh], v[k0 * dh:(k0 + hk_w) * dh]], 0)
    else:
        _copy(ly.kv, fused_qkv(q, k, v, cfg.num_heads, cfg.num_kv_heads, dh, W, r)[model.Hq * dh:], p + "kv")
    _copy(ly.q_w, qs, p + "q_proj")
    _copy(ly.o, o[:, h0 * dh:(h0 + hq_w) * dh], p + "o_proj")


def load_dense_decoder(model, get_tensor: Callable[[str], torch.Tensor], names: set[str],
                       mlp_loader: Callable | None = None):
    """Llama/Qwen-style decoder; ``mlp_loader(model, layer, get_tensor, names, prefix)``
    replaces the dense MLP loading (MoE models)."""
    cfg = model.cfg
    W, r = model.tp.world, model.tp.rank
    pre = "model." if any(n.startswith("model.") for n in names) else ""
    if any(n.startswith("model.language_model.") for n in names):
        pre = "model.language_model."
    # component data parallelism shards the embedding / LM head over its group
    (ew, er, ev), (hw, hr, hv) = _vocab_shards(model, W, r)
    _copy(model.embed, shard_rows(get_tensor(pre + "embed_tokens.weight"), ew, er, ev), "embed")
    for i, ly in enumerate(model.layers):
        p = f"{pre}layers.{i}."
        _copy(ly.input_norm, get_tensor(p + "input_layernorm.weight"), p + "input_layernorm")
        _copy(ly.post_norm, get_tensor(p + "post_attention_layernorm.weight"), p + "post_attention_layernorm")
        q = get_tensor(p + "self_attn.q_proj.weight")
        k = get_tensor(p + "self_attn.k_proj.weight")
        v = get_tensor(p + "self_attn.v_proj.weight")
        if getattr(model, "cdp_attn", False):
            _load_attention_dp(model, ly, q, k, v, get_tensor(p + "self_attn.o_proj.weight"), W, r, p)
            if ly.q_norm is not None:
                _copy(ly.q_norm, get_tensor(p + "self_attn.q_norm.weight"), p + "q_norm")
                _copy(ly.k_norm, get_tensor(p + "self_attn.k_norm.weight"), p + "k_norm")
            if mlp_loader is not None:
                mlp_loader(model, ly, get_tensor, names, p)
            else:
                load_dense_mlp(model, ly, get_tensor, p)
            continue
        _copy(ly.qkv, fused_qkv(q, k, v, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, W, r), p + "qkv")
        if ly.qkv_bias is not None:
            qb = get_tensor(p + "self_attn.q_proj.bias")[:, None]
            kb = get_tensor(p + "self_attn.k_proj.bias")[:, None]
            vb = get_tensor(p + "self_attn.v_proj.bias")[:, None]
            _copy(ly.qkv_bias, fused_qkv(qb, kb, vb, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, W, r)[:, 0], p + "qkv_bias")
        _copy(ly.o, shard_cols(get_tensor(p + "self_attn.o_proj.weight"), W, r), p + "o_proj")
        if ly.q_norm is not None:
            _copy(ly.q_norm, get_tensor(p + "self_attn.q_norm.weight"), p + "q_norm")
            _copy(ly.k_norm, get_tensor(p + "self_attn.k_norm.weight"), p + "k_norm")
        if mlp_loader is not None:
            mlp_loader(model, ly, get_tensor, names, p)
            continue
        load_dense_mlp(model, ly, get_tensor, p)
    _copy(model.final_norm, get_tensor(pre + "norm.weight"), "norm")
    if getattr(model, "lm_head_from_embed", False):  # tied, but sharded differently
        _copy(model.lm_head, shard_rows(get_tensor(pre + "embed_tokens.weight"), hw, hr, hv), "lm_head")
    elif not cfg.tie_word_embeddings:
        head = "lm_head.weight"
        if head in names:
            _copy(model.lm_head, shard_rows(get_tensor(head), hw, hr, hv), "lm_head")
        else:  # encoder-only checkpoints (embedding models) carry no LM head
            model.lm_head = model.embed


def load_dense_mlp(model, ly, get_tensor, p: str):
    """SwiGLU MLP of one layer: gate/up rows sharded (and block-interleaved for the fused SiLU
    epilogue), down columns sharded (over every rank under component data parallelism of the
    MLP, else over TP)."""
    mg = model.cdp_groups["mlp"][1] if getattr(model, "cdp_mlp", False) else model.tp
    W, r = mg.world, mg.rank
    g = shard_rows(get_tensor(p + "mlp.gate_proj.weight"), W, r)
    u = shard_rows(get_tensor(p + "mlp.up_proj.weight"), W, r)
    gu = L.interleave_gate_up(g, u) if model.silu_blk else torch.cat([g, u], 0)
    _copy(ly.gate_up, gu, p + "gate_up")
    _copy(ly.down, shard_cols(get_tensor(p + "mlp.down_proj.weight"), W, r), p + "down_proj")


def _expert_tensor(get_tensor, names, base: str) -> torch.Tensor:
    """An expert weight in bf16 form: ``base`` itself, or ``base_blocks`` + ``base_scales``
    (MXFP4) dequantized."""
    if base in names:
        return get_tensor(base)
    from ..models.gpt_oss import dequant_mxfp4

    return dequant_mxfp4(get_tensor(base + "_blocks"), get_tensor(base + "_scales"))


@torch.no_grad()
def load_gpt_oss(model, get_tensor: Callable[[str], torch.Tensor], names: set[str]):
    """GPT-OSS: attention as the dense decoder (plus sinks and o_proj bias), experts sharded by
    expert index over the TP ranks.  HF stores ``gate_up_proj [E, H, 2I]`` with gate/up
    interleaved in the last dim and ``down_proj [E, I, H]``; MXFP4 checkpoints store the
    ``[E, 2I, H]`` / ``[E, H, I]`` (out, in) matrices as blocks + scales."""
    cfg = model.cfg
    W, r = model.tp.world, model.tp.rank
    pre = "model."
    (ew, er, ev), (hw, hr, hv) = _vocab_shards(model, W, r)
    _copy(model.embed, shard_rows(get_tensor(pre + "embed_tokens.weight"), ew, er, ev), "embed")
    e0, el = model.e_start, model.e_local
    for i, ly in enumerate(model.layers):
        p = f"{pre}layers.{i}."
        _copy(ly.input_norm, get_tensor(p + "input_layernorm.weight"), p + "input_layernorm")
        _copy(ly.post_norm, get_tensor(p + "post_attention_layernorm.weight"), p + "post_attention_layernorm")
        q = get_tensor(p + "self_attn.q_proj.weight")
        k = get_tensor(p + "self_attn.k_proj.weight")
        v = get_tensor(p + "self_attn.v_proj.weight")
        if getattr(model, "cdp_attn", False):
            _load_attention_dp(model, ly, q, k, v, get_tensor(p + "self_attn.o_proj.weight"), W, r, p)
        else:
            _copy(ly.qkv, fused_qkv(q, k, v, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, W, r), p + "qkv")
            _copy(ly.o, shard_cols(get_tensor(p + "self_attn.o_proj.weight"), W, r), p + "o_proj")
        qb = get_tensor(p + "self_attn.q_proj.bias")[:, None]
        kb = get_tensor(p + "self_attn.k_proj.bias")[:, None]
        vb = get_tensor(p + "self_attn.v_proj.bias")[:, None]
        _copy(ly.qkv_bias, fused_qkv(qb, kb, vb, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, W, r)[:, 0],
              p + "qkv_bias")
        _copy(ly.o_bias, get_tensor(p + "self_attn.o_proj.bias"), p + "o_proj.bias")
        sinks = get_tensor(p + "self_attn.sinks").float()
        _copy(ly.sinks, sinks[r * model.Hq:(r + 1) * model.Hq], p + "sinks")
        _copy(ly.router, get_tensor(p + "mlp.router.weight"), p + "router")
        _copy(ly.router_bias, get_tensor(p + "mlp.router.bias").float(), p + "router.bias")
        gu_name = p + "mlp.experts.gate_up_proj"
        if gu_name in names:
            gu = get_tensor(gu_name)[e0:e0 + el].transpose(1, 2)   # [el, 2I, H] interleaved rows
        else:
            gu = _expert_tensor(get_tensor, names, gu_name)[e0:e0 + el]
        gub = get_tensor(gu_name + "_bias")[e0:e0 + el]
        _copy(ly.w_gu, torch.cat([gu[:, 0::2], gu[:, 1::2]], 1), p + "w_gu")
        _copy(ly.b_gu, torch.cat([gub[:, 0::2], gub[:, 1::2]], 1), p + "b_gu")
        dn_name = p + "mlp.experts.down_proj"
        if dn_name in names:
            dn = get_tensor(dn_name)[e0:e0 + el].transpose(1, 2)   # [el, H, I]
        else:
            dn = _expert_tensor(get_tensor, names, dn_name)[e0:e0 + el]
        _copy(ly.w_down, dn, p + "w_down")
        _copy(ly.b_down, get_tensor(dn_name + "_bias")[e0:e0 + el], p + "b_down")
        # MXFP4 checkpoints keep their experts in MXFP4 for decode; bf16 checkpoints stay bf16
        if getattr(model, "use_fp4", False):
            if gu_name + "_blocks" in names:
                gb = get_tensor(gu_name + "_blocks")[e0:e0 + el]
                gs = get_tensor(gu_name + "_scales")[e0:e0 + el]
                model.set_expert_mxfp4(ly, torch.cat([gb[:, 0::2], gb[:, 1::2]], 1),
                                       torch.cat([gs[:, 0::2], gs[:, 1::2]], 1),
                                       get_tensor(dn_name + "_blocks")[e0:e0 + el],
                                       get_tensor(dn_name + "_scales")[e0:e0 + el])
    _copy(model.final_norm, get_tensor(pre + "norm.weight"), "norm")
    _copy(model.lm_head, shard_rows(get_tensor("lm_head.weight"), hw, hr, hv), "lm_head")


@torch.no_grad()
def load_qwen3_5(model, get_tensor: Callable[[str], torch.Tensor], names: set[str]):
    """Hybrid Qwen3.5/3.6 text decoder.  RMSNorm weights are stored as offsets from 1 and are
    converted to scales; linear-attention heads/channels and attention heads are split over
    the TP ranks; experts by index (see :func:`..models.qwen_moe.load_moe_mlp`)."""
    from ..models.qwen_moe import load_moe_mlp

    cfg = model.cfg
    W, r = model.tp.world, model.tp.rank
    pre = "model.language_model." if any(n.startswith("model.language_model.") for n in names) else "model."
    one = lambda t: t.float() + 1.0  # noqa: E731
    (ew, er, ev), (hw, hr, hv) = _vocab_shards(model, W, r)
    _copy(model.embed, shard_rows(get_tensor(pre + "embed_tokens.weight"), ew, er, ev), "embed")
    Hk, Hv, dk, dv = model.lin_Hk, model.lin_Hv, model.lin_dk, model.lin_dv
    Kd, Vd = cfg.linear_num_key_heads * dk, cfg.linear_num_value_heads * dv
    for i, ly in enumerate(model.layers):
        p = f"{pre}layers.{i}."
        _copy(ly.input_norm, one(get_tensor(p + "input_layernorm.weight")), p + "input_layernorm")
        _copy(ly.post_norm, one(get_tensor(p + "post_attention_layernorm.weight")), p + "post_attention_layernorm")
        if model.is_linear[i]:
            a = p + "linear_attn."
            qkv = get_tensor(a + "in_proj_qkv.weight")
            q = qkv[:Kd][r * Hk * dk:(r + 1) * Hk * dk]
            k = qkv[Kd:2 * Kd][r * Hk * dk:(r + 1) * Hk * dk]
            v = qkv[2 * Kd:2 * Kd + Vd][r * Hv * dv:(r + 1) * Hv * dv]
            z = get_tensor(a + "in_proj_z.weight")[r * Hv * dv:(r + 1) * Hv * dv]
            bw = get_tensor(a + "in_proj_b.weight")[r * Hv:(r + 1) * Hv]
            aw = get_tensor(a + "in_proj_a.weight")[r * Hv:(r + 1) * Hv]
            _copy(ly.w_in, torch.cat([q, k, v, z, bw, aw], 0), a + "in_proj")
            cw = get_tensor(a + "conv1d.weight").reshape(2 * Kd + Vd, -1)
            cw = torch.cat([cw[:Kd][r * Hk * dk:(r + 1) * Hk * dk], cw[Kd:2 * Kd][r * Hk * dk:(r + 1) * Hk * dk],
                            cw[2 * Kd:][r * Hv * dv:(r + 1) * Hv * dv]], 0)
            _copy(ly.conv_w, cw, a + "conv1d")
            _copy(ly.A_log, get_tensor(a + "A_log")[r * Hv:(r + 1) * Hv].float(), a + "A_log")
            _copy(ly.dt_bias, get_tensor(a + "dt_bias")[r * Hv:(r + 1) * Hv].float(), a + "dt_bias")
            _copy(ly.gnorm_w, get_tensor(a + "norm.weight"), a + "norm")
            _copy(ly.out_proj, get_tensor(a + "out_proj.weight")[:, r * Hv * dv:(r + 1) * Hv * dv], a + "out_proj")
        else:
            a = p + "self_attn."
            D = cfg.head_dim
            qg = get_tensor(a + "q_proj.weight").view(cfg.num_heads, 2, D, -1)
            qw, gw = qg[:, 0].reshape(cfg.num_heads * D, -1), qg[:, 1].reshape(cfg.num_heads * D, -1)
            qkv = fused_qkv(qw, get_tensor(a + "k_proj.weight"), get_tensor(a + "v_proj.weight"),
                            cfg.num_heads, cfg.num_kv_heads, D, W, r)
            gate = gw[r * model.Hq * D:(r + 1) * model.Hq * D]
            _copy(ly.qkvg, torch.cat([qkv, gate], 0), a + "qkvg")
            _copy(ly.q_norm, one(get_tensor(a + "q_norm.weight")), a + "q_norm")
            _copy(ly.k_norm, one(get_tensor(a + "k_norm.weight")), a + "k_norm")
            _copy(ly.o, shard_cols(get_tensor(a + "o_proj.weight"), W, r), a + "o_proj")
        load_moe_mlp(model, ly, get_tensor, names, p)
    _copy(model.final_norm, one(get_tensor(pre + "norm.weight")), "norm")
    if cfg.tie_word_embeddings:
        return
    _copy(model.lm_head, shard_rows(get_tensor("lm_head.weight"), hw, hr, hv), "lm_head")


_VIS_ATTR = {"attn.qkv.weight": "qkv_w", "attn.qkv.bias": "qkv_b", "attn.proj.weight": "proj_w",
             "mlp.linear_fc1.weight": "fc1_w", "mlp.linear_fc1.bias": "fc1_b",
             "mlp.linear_fc2.weight": "fc2_w"}
_VIS_ATTR = collections.defaultdict(lambda: "replicated", _VIS_ATTR)


@torch.no_grad()
def load_qwen3_vl_vision(vis, get_tensor: Callable[[str], torch.Tensor], names: set[str]):
    """Qwen3-VL vision encoder: Conv3d patch embedding flattened to a linear layer, position
    table, blocks (attention heads and MLP sharded over the vision TP group, if any), merger
    and DeepStack mergers (replicated)."""
    pre = "model.visual." if any(n.startswith("model.visual.") for n in names) else "visual."
    w = get_tensor(pre + "patch_embed.proj.weight")
    _copy(vis.patch_w, w.reshape(w.shape[0], -1), "patch_embed")
    _copy(vis.patch_b, get_tensor(pre + "patch_embed.proj.bias"), "patch_embed.bias")
    _copy(vis.pos_embed, get_tensor(pre + "pos_embed.weight"), "pos_embed")
    for i, blk in enumerate(vis.blocks):
        p = f"{pre}blocks.{i}."
        for dst, src in ((blk.n1_w, "norm1.weight"), (blk.n1_b, "norm1.bias"), (blk.n2_w, "norm2.weight"),
                         (blk.n2_b, "norm2.bias"), (blk.qkv_w, "attn.qkv.weight"), (blk.qkv_b, "attn.qkv.bias"),
                         (blk.proj_w, "attn.proj.weight"), (blk.proj_b, "attn.proj.bias"),
                         (blk.fc1_w, "mlp.linear_fc1.weight"), (blk.fc1_b, "mlp.linear_fc1.bias"),
                         (blk.fc2_w, "mlp.linear_fc2.weight"), (blk.fc2_b, "mlp.linear_fc2.bias")):
            _copy(dst, vis.shard(p + _VIS_ATTR[src], get_tensor(p + src)), p + src)
    mergers = [(vis.merger, pre + "merger.")] + [(m, f"{pre}deepstack_merger_list.{j}.")
                                                   for j, m in enumerate(vis.deep_mergers)]
    for m, p in mergers:
        for dst, src in ((m.n_w, "norm.weight"), (m.n_b, "norm.bias"), (m.fc1_w, "linear_fc1.weight"),
                         (m.fc1_b, "linear_fc1.bias"), (m.fc2_w, "linear_fc2.weight"),
                         (m.fc2_b, "linear_fc2.bias")):
            _copy(dst, get_tensor(p + src), p + src)
