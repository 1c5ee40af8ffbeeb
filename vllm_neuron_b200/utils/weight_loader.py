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
def load_dense_decoder(model, get_tensor: Callable[[str], torch.Tensor], names: set[str]):
    cfg = model.cfg
    W, r = model.tp.world, model.tp.rank
    pre = "model." if any(n.startswith("model.") for n in names) else ""
    if any(n.startswith("model.language_model.") for n in names):
        pre = "model.language_model."
    _copy(model.embed, shard_rows(get_tensor(pre + "embed_tokens.weight"), W, r, model.V_local), "embed")
    for i, ly in enumerate(model.layers):
        p = f"{pre}layers.{i}."
        _copy(ly.input_norm, get_tensor(p + "input_layernorm.weight"), p + "input_layernorm")
        _copy(ly.post_norm, get_tensor(p + "post_attention_layernorm.weight"), p + "post_attention_layernorm")
        q = get_tensor(p + "self_attn.q_proj.weight")
        k = get_tensor(p + "self_attn.k_proj.weight")
        v = get_tensor(p + "self_attn.v_proj.weight")
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
        g = shard_rows(get_tensor(p + "mlp.gate_proj.weight"), W, r)
        u = shard_rows(get_tensor(p + "mlp.up_proj.weight"), W, r)
        gu = L.interleave_gate_up(g, u) if model.silu_blk else torch.cat([g, u], 0)
        _copy(ly.gate_up, gu, p + "gate_up")
        _copy(ly.down, shard_cols(get_tensor(p + "mlp.down_proj.weight"), W, r), p + "down_proj")
    _copy(model.final_norm, get_tensor(pre + "norm.weight"), "norm")
    if not cfg.tie_word_embeddings:
        head = "lm_head.weight"
        _copy(model.lm_head, shard_rows(get_tensor(head), W, r, model.V_local), "lm_head")
