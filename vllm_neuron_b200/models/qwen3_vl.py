"""Qwen3-VL (``Qwen3VLForConditionalGeneration``): a Qwen3 text decoder with interleaved
multimodal RoPE and DeepStack visual features, plus a ViT image encoder.

Vision encoder (``Qwen3VLVision``, replicated on every TP rank):

    patches [N, C * Tp * P * P] -> linear patch embedding (+ bias)
      + learned position table bilinearly interpolated to the image grid
    depth x block: x += proj(attn(LN1(x)))   (full attention inside each image, 2-D rotary
                                              embedding of the (row, column) patch position)
                   x += fc2(gelu_tanh(fc1(LN2(x))))
    merger: LN -> group 2 x 2 neighbouring patches -> fc1 -> GELU -> fc2  => text hidden size
    DeepStack: after the blocks listed in ``deepstack_visual_indexes`` a merger of the same
    form (LayerNorm after the grouping) produces features that are added to the text residual
    stream at the image-token rows after decoder layers 0, 1, ...

Text decoder: :class:`.llama.LlamaForCausalLM` with QK-norm; image-token rows take the merged
vision embeddings (the prompt-embedding path of the runner) and rotate with 3-D positions
(temporal, row, column) through the interleaved M-RoPE of the rope kernel; text tokens use
(p, p, p), which equals the 1-D rotation, shifted by the request's position delta after an
image.

Reference: vllm_neuron/model/qwen3_vl/model_bf16.py, vision_encoder_bf16.py,
utils/mrope.py (3-D positions), utils/merge_vision_embeds.py; the math follows the published
Qwen3-VL definition (HF ``Qwen3VLForConditionalGeneration``).  The vision encoder runs its
linear layers on the tcgen05 GEMM; its LayerNorm, GELU and per-image attention use torch ops.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from ..ops import linear as L
from ..parallel.comm import SINGLE, GroupComm
from . import vision_packing as VP
from .llama import LlamaForCausalLM


def _lin(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    if isinstance(w, L.MXFP8Weight):  # MXFP8 vision weights (block-scaled tensor cores / oracle)
        y = L.gemm_out(x.contiguous(), w) if x.shape[0] > 0 else x.new_zeros(0, w.shape[0])
        return (y + b if b is not None else y).to(x.dtype)
    if x.is_cuda and x.dtype == torch.bfloat16 and x.shape[0] > 0:
        y = L.gemm_out(x.contiguous(), w)
    else:
        y = (x.float() @ w.float().t()).to(x.dtype)
    return y + b if b is not None else y


class Qwen3VLVision(torch.nn.Module):
    """Qwen3-VL vision encoder.  With a vision TP group of ``V`` ranks each block's attention
    heads and MLP are sharded (qkv / fc1 by output rows, proj / fc2 by input columns, followed
    by an all-reduce; reference: the vision TP group, vllm_neuron/parallel/
    neuron_parallel_state.py:667-701, model/qwen3_vl/vision_encoder_bf16.py:156,355,623)."""

    SHARD_ROWS = ("qkv_w", "qkv_b", "fc1_w", "fc1_b")   # output-sharded block parameters
    SHARD_COLS = ("proj_w", "fc2_w")                    # input-sharded block parameters

    def __init__(self, vc: dict, device, dtype, tp: GroupComm = SINGLE):
        super().__init__()
        self.tp = tp
        self.hidden = vc["hidden_size"]
        self.heads = vc["num_heads"]
        self.depth = vc["depth"]
        self.inter = vc["intermediate_size"]
        self.patch = vc.get("patch_size", 16)
        self.tpatch = vc.get("temporal_patch_size", 2)
        self.in_ch = vc.get("in_channels", 3)
        self.merge = vc.get("spatial_merge_size", 2)
        self.out_hidden = vc["out_hidden_size"]
        self.num_pos = vc.get("num_position_embeddings", 2304)
        self.grid_side = int(round(math.sqrt(self.num_pos)))
        self.deep_idx = list(vc.get("deepstack_visual_indexes") or [])
        self.act = vc.get("hidden_act", "gelu_pytorch_tanh")
        h, hm = self.hidden, self.hidden * self.merge ** 2
        V = tp.world
        if self.heads % V or self.inter % V:
            raise ValueError(f"vision TP={V} must divide the vision heads ({self.heads}) and "
                             f"the MLP width ({self.inter})")
        self.heads_l, self.inter_l = self.heads // V, self.inter // V
        hl = h // V
        kw = dict(device=device, dtype=dtype)

        def P(*shape):
            return torch.nn.Parameter(torch.zeros(*shape, **kw), requires_grad=False)

        self.patch_w = P(h, self.in_ch * self.tpatch * self.patch * self.patch)
        self.patch_b = P(h)
        self.pos_embed = P(self.num_pos, h)
        self.blocks = torch.nn.ModuleList()
        for _ in range(self.depth):
            m = torch.nn.Module()
            m.n1_w, m.n1_b, m.n2_w, m.n2_b = P(h), P(h), P(h), P(h)
            m.qkv_w, m.qkv_b = P(3 * hl, h), P(3 * hl)
            m.proj_w, m.proj_b = P(h, hl), P(h)
            m.fc1_w, m.fc1_b = P(self.inter_l, h), P(self.inter_l)
            m.fc2_w, m.fc2_b = P(h, self.inter_l), P(h)
            self.blocks.append(m)

        def merger(post_norm: bool):
            m = torch.nn.Module()
            m.post_norm = post_norm
            m.n_w, m.n_b = P(hm if post_norm else h), P(hm if post_norm else h)
            m.fc1_w, m.fc1_b = P(hm, hm), P(hm)
            m.fc2_w, m.fc2_b = P(self.out_hidden, hm), P(self.out_hidden)
            return m

        self.merger = merger(False)
        self.deep_mergers = torch.nn.ModuleList([merger(True) for _ in self.deep_idx])
        hd = h // self.heads
        self.rot_inv_freq = 1.0 / (10000.0 ** (torch.arange(0, hd // 2, 2, dtype=torch.float32) / (hd // 2)))

    def shard(self, name: str, full: torch.Tensor) -> torch.Tensor:
        """This rank's slice of the unsharded block parameter ``full`` (``name`` ends with the
        attribute name): q / k / v rows of the local heads, local MLP rows, or the matching
        input columns of proj / fc2."""
        V, r = self.tp.world, self.tp.rank
        attr = name.rsplit(".", 1)[-1]
        if V == 1 or (attr not in self.SHARD_ROWS and attr not in self.SHARD_COLS):
            return full
        if attr.startswith("qkv"):
            h = self.hidden
            hl = h // V
            return full.view(3, h, *full.shape[1:])[:, r * hl:(r + 1) * hl].reshape(3 * hl, *full.shape[1:])
        if attr in self.SHARD_ROWS:
            n = full.shape[0] // V
            return full[r * n:(r + 1) * n]
        n = full.shape[1] // V
        return full[:, r * n:(r + 1) * n]

    def full_shape(self, name: str, local: torch.Tensor) -> tuple:
        attr = name.rsplit(".", 1)[-1]
        V = self.tp.world
        if attr in self.SHARD_ROWS:
            return (local.shape[0] * V,) + tuple(local.shape[1:])
        if attr in self.SHARD_COLS:
            return (local.shape[0], local.shape[1] * V)
        return tuple(local.shape)

    def _row_parallel(self, y: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        """``y @ w.T + b`` with ``w`` sharded by input columns: partial sums all-reduced over
        the vision TP group, the bias added once."""
        if self.tp.world == 1:
            return _lin(y, w, b)
        part = _lin(y, w, None)
        self.tp.all_reduce_(part)
        return part + b

    # ---------------------------------------------------------------- position helpers
    def _pos_embed(self, grids: list[tuple[int, int, int]]) -> torch.Tensor:
        """Learned position table bilinearly resampled to each grid, in merge-block order."""
        dev = self.pos_embed.device
        out = []
        n = self.grid_side
        for t, h, w in grids:
            hi = torch.linspace(0, n - 1, h)
            wi = torch.linspace(0, n - 1, w)
            h0, w0 = hi.int(), wi.int()
            h1, w1 = (h0 + 1).clamp(max=n - 1), (w0 + 1).clamp(max=n - 1)
            dh, dw = hi - h0, wi - w0
            idx = [(h0[:, None] * n + w0[None]), (h0[:, None] * n + w1[None]),
                   (h1[:, None] * n + w0[None]), (h1[:, None] * n + w1[None])]
            wts = [(1 - dh)[:, None] * (1 - dw)[None], (1 - dh)[:, None] * dw[None],
                   dh[:, None] * (1 - dw)[None], dh[:, None] * dw[None]]
            pe = sum(self.pos_embed[i.flatten().to(dev)].float() * wt.flatten()[:, None].to(dev)
                     for i, wt in zip(idx, wts)).to(self.pos_embed.dtype)
            m = self.merge
            pe = pe.repeat(t, 1).view(t, h // m, m, w // m, m, -1).permute(0, 1, 3, 2, 4, 5).reshape(t * h * w, -1)
            out.append(pe)
        return torch.cat(out)

    def _rotary(self, grids) -> tuple[torch.Tensor, torch.Tensor]:
        """cos / sin [N, head_dim] of the 2-D (row, column) rotary embedding, merge-block order."""
        m = self.merge
        rows, cols = [], []
        for t, h, w in grids:
            br = torch.arange(h // m)[:, None, None, None] * m + torch.arange(m)[None, None, :, None]
            bc = torch.arange(w // m)[None, :, None, None] * m + torch.arange(m)[None, None, None, :]
            r = br.expand(h // m, w // m, m, m).reshape(-1)
            c = bc.expand(h // m, w // m, m, m).reshape(-1)
            rows.append(r.repeat(t))
            cols.append(c.repeat(t))
        r, c = torch.cat(rows).float(), torch.cat(cols).float()
        f = torch.cat([r[:, None] * self.rot_inv_freq[None], c[:, None] * self.rot_inv_freq[None]], 1)
        emb = torch.cat([f, f], 1)
        dev = self.pos_embed.device
        return emb.cos().to(dev), emb.sin().to(dev)

    # ---------------------------------------------------------------- forward
    def _act(self, x: torch.Tensor) -> torch.Tensor:
        return F.gelu(x, approximate="tanh") if "tanh" in self.act else F.gelu(x)

    def _merge(self, m, x: torch.Tensor) -> torch.Tensor:
        hm = self.hidden * self.merge ** 2
        if m.post_norm:
            x = F.layer_norm(x.view(-1, hm).float(), (hm,), m.n_w.float(), m.n_b.float(), 1e-6).to(x.dtype)
        else:
            x = F.layer_norm(x.float(), (self.hidden,), m.n_w.float(), m.n_b.float(), 1e-6).to(x.dtype).view(-1, hm)
        x = F.gelu(_lin(x, m.fc1_w, m.fc1_b).float()).to(x.dtype)
        return _lin(x, m.fc2_w, m.fc2_b)

    def _body(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, attend):
        """The encoder blocks and mergers over rows ``x [R, H]`` (rotary ``cos`` / ``sin``
        ``[R, head_dim]``); ``attend(q, k, v)`` maps ``[R, heads, hd]`` bf16 tensors to the
        attention output ``[R, heads * hd]``.  Returns (merged ``[R / merge^2, out_hidden]``,
        DeepStack ``[n_deep, R / merge^2, out_hidden]``)."""
        dt = self.patch_b.dtype
        H, nh = self.hidden, self.heads_l
        hd = H // self.heads
        deep = []
        c, s = cos[:, None, :], sin[:, None, :]
        for li, blk in enumerate(self.blocks):
            y = F.layer_norm(x.float(), (H,), blk.n1_w.float(), blk.n1_b.float(), 1e-6).to(dt)
            qkv = _lin(y, blk.qkv_w, blk.qkv_b).view(-1, 3, nh, hd).float()
            q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
            q = q * c + torch.cat([-q[..., hd // 2:], q[..., :hd // 2]], -1) * s
            k = k * c + torch.cat([-k[..., hd // 2:], k[..., :hd // 2]], -1) * s
            x = x + self._row_parallel(attend(q.to(dt), k.to(dt), v.to(dt)), blk.proj_w, blk.proj_b)
            y = F.layer_norm(x.float(), (H,), blk.n2_w.float(), blk.n2_b.float(), 1e-6).to(dt)
            y = self._act(_lin(y, blk.fc1_w, blk.fc1_b).float()).to(dt)
            x = x + self._row_parallel(y, blk.fc2_w, blk.fc2_b)
            if li in self.deep_idx:
                deep.append(self._merge(self.deep_mergers[self.deep_idx.index(li)], x))
        emb = self._merge(self.merger, x)
        deep_t = torch.stack(deep) if deep else emb.new_zeros(0, emb.shape[0], emb.shape[1])
        return emb, deep_t

    def _embed(self, pixels: torch.Tensor, grids: list[tuple[int, int, int]]):
        """Patch embedding + interpolated position table, and the rotary tables (flat rows)."""
        dt = self.patch_b.dtype
        x = _lin(pixels.to(self.patch_b.device, dt), self.patch_w, self.patch_b)
        x = x + self._pos_embed(grids)
        cos, sin = self._rotary(grids)
        return x, cos, sin

    @torch.no_grad()
    def forward(self, pixels: torch.Tensor, grids: list[tuple[int, int, int]]):
        """``pixels [N, C * Tp * P * P]`` -> (embeds ``[N / merge^2, out_hidden]``, DeepStack
        features ``[len(deepstack), N / merge^2, out_hidden]``).  Attention runs separately
        for every frame of every image (one call per frame)."""
        x, cos, sin = self._embed(pixels, grids)
        frames = [h * w for t, h, w in grids for _ in range(t)]

        def attend(q, k, v):
            outs, o0 = [], 0
            for n in frames:
                qi, ki, vi = (z[o0:o0 + n].transpose(0, 1)[None] for z in (q, k, v))
                outs.append(F.scaled_dot_product_attention(qi, ki, vi)[0].transpose(0, 1).reshape(n, -1))
                o0 += n
            return torch.cat(outs)

        return self._body(x, cos, sin, attend)

    def packed_body(self, xp: torch.Tensor, cp: torch.Tensor, sp: torch.Tensor,
                    mask: torch.Tensor):
        """Encoder over packed blocks: ``xp [B * bs, H]`` rows in ``B = mask.shape[0]`` blocks,
        attention of all blocks in one batched call restricted by ``mask [B, 1, bs, bs]``.
        Shapes depend on ``(B, bs)`` only, so one CUDA graph serves every plan of that size."""
        B, bs = mask.shape[0], mask.shape[-1]

        def attend(q, k, v):
            nh, hd = q.shape[1], q.shape[2]
            qb, kb, vb = (z.view(B, bs, nh, hd).transpose(1, 2) for z in (q, k, v))
            o = F.scaled_dot_product_attention(qb, kb, vb, attn_mask=mask)
            return o.transpose(1, 2).reshape(B * bs, nh * hd)

        return self._body(xp, cp, sp, attend)

    @torch.no_grad()
    def forward_packed(self, pixels: torch.Tensor, grids: list[tuple[int, int, int]],
                       plan: "VP.PackPlan", body=None):
        """Same result as :meth:`forward` with the images' patches packed into the blocks of
        ``plan`` (one item per image, in image order).  ``body`` replaces :meth:`packed_body`
        (a CUDA-graph replay of it)."""
        x, cos, sin = self._embed(pixels, grids)
        dev = x.device
        dst = VP.scatter_index(plan).to(dev)
        xp, cp, sp = (VP.to_blocks(z, plan, dst) for z in (x, cos, sin))
        lo, hi = VP.block_bounds(plan, frames=[t for t, _, _ in grids])
        mask = VP.bounds_mask(lo.to(dev), hi.to(dev))
        emb, deep = (body or self.packed_body)(xp, cp, sp, mask)
        idx = VP.unpack_index(plan, self.merge ** 2).to(dev)
        return emb.index_select(0, idx), deep.index_select(1, idx)


@torch.no_grad()
def quantize_vision_mxfp8(v: "Qwen3VLVision") -> int:
    """Turn the vision encoder's linear weights whose input width is a multiple of 128 (patch
    embedding, block qkv / proj / fc1 / fc2, merger fc1 / fc2) into MXFP8 weights; returns how
    many were converted."""
    mods = [(v, ("patch_w",))] + [(blk, ("qkv_w", "proj_w", "fc1_w", "fc2_w")) for blk in v.blocks]
    mods += [(m, ("fc1_w", "fc2_w")) for m in [v.merger, *v.deep_mergers]]
    n = 0
    for mod, names in mods:
        for name in names:
            w = getattr(mod, name)
            if not isinstance(w, torch.Tensor) or w.dim() != 2 or w.shape[1] % 128:
                continue
            mw = L.MXFP8Weight.from_weight(w)
            if name in mod._parameters:
                del mod._parameters[name]
            setattr(mod, name, mw)
            n += 1
    return n


def mrope_positions(prompt: list[int], image_token_id, grids: list[tuple[int, int, int]],
                    merge: int) -> tuple[np.ndarray, int]:
    """3-D positions ``[3, P]`` of a prompt whose image placeholders are already expanded, and
    the position delta of the tokens after the prompt (``pos = index + delta``).  Text tokens
    count up by one; an image of grid (t, h, w) occupies (t h w) / merge^2 tokens at
    (start, start + row, start + col) and advances the counter by max(h, w) / merge."""
    vis = set(image_token_id) if isinstance(image_token_id, (set, list, tuple)) else {image_token_id}
    P = len(prompt)
    pos = np.zeros((3, P), dtype=np.int64)
    cur = 0
    i = 0
    g = iter(grids)
    while i < P:
        if prompt[i] not in vis:
            pos[:, i] = cur
            cur += 1
            i += 1
            continue
        t, h, w = next(g)
        gh, gw = h // merge, w // merge
        n = t * gh * gw
        if prompt[i:i + n] != [prompt[i]] * n:
            raise ValueError("image placeholder count does not match the image grid")
        pos[0, i:i + n] = cur
        pos[1, i:i + n] = cur + np.repeat(np.arange(gh), gw * t)
        pos[2, i:i + n] = cur + np.tile(np.arange(gw), gh * t)
        cur += max(h, w) // merge
        i += n
    delta = int(pos.max()) + 1 - P if P else 0
    return pos, delta


class Qwen3VLForConditionalGeneration(LlamaForCausalLM):
    supports_prefix_caching = False  # image tokens share ids: cached blocks would not match pixels

    def __init__(self, cfg, *args, **kw):
        super().__init__(cfg, *args, **kw)
        raw = cfg.raw
        vc = dict(raw.get("vision_config") or {})
        vc.setdefault("out_hidden_size", self.H)
        self.visual_config = vc
        self.visual = Qwen3VLVision(vc, self.device, self.dtype)
        rp = (raw.get("rope_parameters") or raw.get("rope_scaling") or {})
        sec = rp.get("mrope_section") or [24, 20, 20]
        self.mrope_section = (int(sec[0]), int(sec[1]), int(sec[2]))
        self.image_token_id = int(raw.get("image_token_id", 151655))
        self.video_token_id = int(raw.get("video_token_id", 151656))
        self.spatial_merge = self.visual.merge

    @torch.no_grad()
    def init_random(self, seed: int = 0, std: float = 0.02):
        super().init_random(seed, std)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 1000 + 17)
        for name, prm in self.visual.named_parameters():
            if name.endswith("_w") and ("n1" in name or "n2" in name or name.startswith("n_") or ".n_" in name):
                prm.fill_(1.0)
            elif name.endswith("_b"):
                prm.zero_()
            else:  # drawn at full size, then sharded: the same weights for every vision TP size
                full = torch.empty(self.visual.full_shape(name, prm), dtype=prm.dtype, device=prm.device)
                full.normal_(0.0, std, generator=g)
                prm.copy_(self.visual.shard(name, full))

    def set_vision_tp(self, group: GroupComm):
        """Rebuild the (not yet loaded) vision encoder sharded over ``group``: consecutive TP
        ranks; the TP group then holds TP / V vision-DP replicas."""
        vc = self.visual_config
        self.visual = Qwen3VLVision(vc, self.device, self.dtype, tp=group)

    vision_dp = True  # split a request's images over the TP ranks (vision data parallelism)
    vision_calls = 0  # images encoded by this rank (observability / tests)
    vision_pack = None  # VisionConfig: images packed into blocks (None: one call per image)
    vision_graphs = False
    vision_blocks = 0   # packed blocks encoded by this rank

    def configure_vision(self, vcfg, cuda_graphs: bool = True):
        """Run the encoder on packed blocks of ``vcfg.vision_attention_block_size`` rows with
        the block counts of ``vcfg.num_vision_tokens_buckets``; on the GPU (vision TP 1) each
        block count's encoder forward is a CUDA graph captured on first use."""
        if vcfg.vision_attention_block_size % (self.spatial_merge ** 2):
            raise ValueError("vision_attention_block_size must be a multiple of the merge group")
        self.vision_pack = vcfg
        self.vision_graphs = bool(cuda_graphs and vcfg.cuda_graphs and self.device.type == "cuda"
                                  and self.visual.tp.world == 1)
        self._vgraphs: dict[tuple[int, int], tuple] = {}
        self._vgraph_pool = None

    def _capture_vision(self, nb: int, bs: int):
        """CUDA graph of :meth:`Qwen3VLVision.packed_body` for ``nb`` blocks of ``bs`` rows:
        (graph, static inputs, static outputs)."""
        vis, dev = self.visual, self.device
        R, hd = nb * bs, vis.hidden // vis.heads
        ins = (torch.zeros(R, vis.hidden, dtype=vis.patch_b.dtype, device=dev),
               torch.ones(R, hd, dtype=torch.float32, device=dev),
               torch.zeros(R, hd, dtype=torch.float32, device=dev),
               torch.ones(nb, 1, bs, bs, dtype=torch.bool, device=dev))
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            vis.packed_body(*ins)  # warm-up: allocator, kernel selection
        torch.cuda.current_stream(dev).wait_stream(side)
        if self._vgraph_pool is None:
            self._vgraph_pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self._vgraph_pool):
            outs = vis.packed_body(*ins)
        return g, ins, outs

    def _packed_runner(self, nb: int, bs: int):
        if not self.vision_graphs:
            return self.visual.packed_body
        ent = self._vgraphs.get((nb, bs))
        if ent is None:
            ent = self._vgraphs[(nb, bs)] = self._capture_vision(nb, bs)
        g, ins, outs = ent

        def run(xp, cp, sp, mask):
            for dst, src in zip(ins, (xp, cp, sp, mask)):
                dst.copy_(src)
            g.replay()
            return outs
        return run

    def _encode_packed(self, pixels: torch.Tensor, grids: list[tuple[int, int, int]]):
        """:meth:`encode_images` on packed blocks.  With vision data parallelism the block count
        is padded to the ``W`` replicas, replica ``r`` encodes blocks ``[r * nb, (r + 1) * nb)``
        and the merged rows are all-gathered before they are put back in image order.
        Returns None when an image does not fit a block (the caller encodes per image)."""
        vis, vc = self.visual, self.vision_pack
        V = vis.tp.world
        W = self.tp.world // V if self.vision_dp else 1
        bs = vc.vision_attention_block_size
        sizes = [t * h * w for t, h, w in grids]
        if max(sizes) > bs:
            return None
        try:
            plan = VP.plan_for_buckets(sizes, bs, vc.num_vision_tokens_buckets, dp=W)
        except ValueError:  # more tokens than the largest bucket: the minimal plan, uncaptured
            plan = VP.plan_for_buckets(sizes, bs, None, dp=W)
        x, cos, sin = vis._embed(pixels, grids)
        dev = x.device
        dst = VP.scatter_index(plan).to(dev)
        lo, hi = VP.block_bounds(plan, frames=[t for t, _, _ in grids])
        nb = plan.num_blocks // W
        r = self.tp.rank // V if W > 1 else 0
        rows = slice(r * nb * bs, (r + 1) * nb * bs)
        xp, cp, sp = (VP.to_blocks(z, plan, dst)[rows] for z in (x, cos, sin))
        mask = VP.bounds_mask(lo[r * nb:(r + 1) * nb].to(dev), hi[r * nb:(r + 1) * nb].to(dev))
        emb, deep = self._packed_runner(nb, bs)(xp, cp, sp, mask)
        self.vision_blocks += nb
        H, nd = self.H, len(vis.deep_idx)
        if W > 1:
            n = emb.shape[0]
            parts = [emb] + ([deep.permute(1, 0, 2).reshape(n, nd * H)] if nd else [])
            allp = self.tp.all_gather(torch.cat(parts, 1).unsqueeze(0), dim=0)  # [W * V, n, .]
            allp = allp.view(W, V, n, -1)[:, 0].reshape(W * n, -1)  # each replica's first rank
            emb = allp[:, :H]
            deep = (allp[:, H:].reshape(W * n, nd, H).permute(1, 0, 2) if nd
                    else emb.new_zeros(0, W * n, H))
        idx = VP.unpack_index(plan, self.spatial_merge ** 2).to(dev)
        return emb.index_select(0, idx), deep.index_select(1, idx).contiguous()

    def encode_images(self, pixels: torch.Tensor, grids: list[tuple[int, int, int]]):
        """Merged vision embeddings ``[tokens, H]`` and DeepStack features ``[n_deep, tokens, H]``
        of the images of one request, in image order.

        Vision data parallelism: with TP > 1 and several images, image ``i`` is encoded by TP
        rank ``i % W`` only (the vision weights are replicated) and the results are all-gathered
        (padded to the largest share), instead of every rank encoding every image.  Reference:
        the vision TP/DP groups (vllm_neuron/parallel/neuron_parallel_state.py:667-701; vision
        DP defaults to the world, vllm_neuron/model/neuron_config.py:345-404)."""
        if self.vision_pack is not None:
            res = self._encode_packed(pixels, grids)
            if res is not None:
                self.vision_calls += len(grids)
                return res
        V = self.visual.tp.world
        W = self.tp.world // V   # vision-DP replicas of V consecutive ranks
        if W == 1 or len(grids) < 2 or not self.vision_dp:
            self.vision_calls += len(grids)
            return self.visual(pixels, grids)
        replica = self.tp.rank // V
        m2 = self.spatial_merge ** 2
        counts = [t * h * w for t, h, w in grids]
        starts = [sum(counts[:i]) for i in range(len(grids))]
        rows = [c // m2 for c in counts]
        owner = [i % W for i in range(len(grids))]
        mine = [i for i in range(len(grids)) if owner[i] == replica]
        H = self.H
        if mine:
            px = torch.cat([pixels[starts[i]:starts[i] + counts[i]] for i in mine])
            emb, deep = self.visual(px, [grids[i] for i in mine])
            self.vision_calls += len(mine)
        else:
            emb, deep = pixels.new_zeros(0, H, dtype=self.dtype), None
        nd = len(self.visual.deep_idx)  # same on every rank, also those without an image
        share = [sum(rows[i] for i in range(len(grids)) if owner[i] == r) for r in range(W)]
        R = max(share)
        pack = torch.zeros(R, H * (1 + nd), dtype=emb.dtype, device=emb.device)
        n = emb.shape[0]
        pack[:n, :H] = emb
        if nd:
            pack[:n, H:] = deep.permute(1, 0, 2).reshape(n, nd * H).to(emb.dtype)
        allp = self.tp.all_gather(pack.unsqueeze(0), dim=0)  # [W * V, R, H * (1 + nd)]
        offs = [0] * W
        e_parts, d_parts = [], []
        for i in range(len(grids)):
            r = owner[i]
            blk = allp[r * V, offs[r]:offs[r] + rows[i]]  # the replica's first rank
            offs[r] += rows[i]
            e_parts.append(blk[:, :H])
            if nd:
                d_parts.append(blk[:, H:].reshape(rows[i], nd, H))
        emb_all = torch.cat(e_parts)
        deep_all = (torch.cat(d_parts).permute(1, 0, 2).contiguous() if nd
                    else emb_all.new_zeros(0, emb_all.shape[0], H))
        return emb_all, deep_all

    @torch.no_grad()
    def quantize_mxfp8(self) -> int:
        """MXFP8 for the text decoder (see the Llama model) and for the vision encoder's linear
        layers whose input width is a multiple of 128: patch embedding, every block's qkv /
        proj / fc1 / fc2 and the mergers' fc1 / fc2 (vision TP shards are quantized as
        loaded).  Reference: the MXFP8 Qwen3-VL (vllm_neuron/model/qwen3_vl/model_mxfp8.py,
        weight_loaders_mxfp8.py)."""
        n = super().quantize_mxfp8() + quantize_vision_mxfp8(self.visual)
        self.mx_linears = n
        return n

    def load_hf_state_dict(self, get_tensor, names: set[str]):
        from ..utils.weight_loader import load_dense_decoder, load_qwen3_vl_vision

        load_dense_decoder(self, get_tensor, names)
        load_qwen3_vl_vision(self.visual, get_tensor, names)
