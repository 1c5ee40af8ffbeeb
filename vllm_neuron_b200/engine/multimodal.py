"""Image inputs of vision-language requests.

``prepare_image_request`` turns a prompt (token ids with one image placeholder per image) plus
images into the model's inputs: the images are resized and patchified by the HF image
processor of the model family (CPU preprocessing, like tokenisation), each placeholder is
expanded to the image's token count, and the 3-D M-RoPE positions and the position delta of
the generated tokens are computed.  The vision encoder runs on the device when the request's
first prefill chunk is scheduled; its output stays with the request until the prompt is
fully prefilled (the encoder cache; reference: EncoderCacheBlocks,
vllm_neuron/vllm/worker/encoder_cache_blocks.py:45-448).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class MultiModalInputs:
    pixels: torch.Tensor                 # [N, C * Tp * P * P] patchified pixels (CPU)
    grids: list                          # [(t, h, w)] patch grid per image
    positions3: np.ndarray               # [3, P] M-RoPE positions of the prompt
    delta: int                           # position offset of tokens after the prompt
    image_rows: np.ndarray               # prompt indexes of the image tokens (in order)
    emb: torch.Tensor | None = None      # device: merged vision embeddings [n_image_tokens, H]
    deep: torch.Tensor | None = None     # device: DeepStack features [n_deep, n_image_tokens, H]
    row_of: dict = field(default_factory=dict)  # prompt index -> image token index


def _processor(model_dir: str | None, vc: dict, overrides: dict | None):
    from transformers.models.qwen2_vl.image_processing_qwen2_vl import Qwen2VLImageProcessor

    kw = dict(patch_size=vc.get("patch_size", 16), temporal_patch_size=vc.get("temporal_patch_size", 2),
              merge_size=vc.get("spatial_merge_size", 2), image_mean=[0.5, 0.5, 0.5], image_std=[0.5, 0.5, 0.5])
    if model_dir and os.path.exists(os.path.join(model_dir, "preprocessor_config.json")):
        with open(os.path.join(model_dir, "preprocessor_config.json")) as f:
            pc = json.load(f)
        for k in ("image_mean", "image_std", "min_pixels", "max_pixels", "patch_size", "merge_size",
                  "temporal_patch_size"):
            if k in pc:
                kw[k] = pc[k]
        if isinstance(pc.get("size"), dict):
            kw["size"] = pc["size"]
    kw.update(overrides or {})
    if "min_pixels" in kw or "max_pixels" in kw:
        kw["size"] = {"shortest_edge": kw.pop("min_pixels", 56 * 56), "longest_edge": kw.pop("max_pixels", 28 * 28 * 1280)}
    return Qwen2VLImageProcessor(**kw)


def _video_processor(model_dir: str | None, vc: dict, overrides: dict | None):
    from transformers.models.qwen3_vl.video_processing_qwen3_vl import Qwen3VLVideoProcessor

    ip = _processor(model_dir, vc, overrides)  # same geometry and normalisation as images
    return Qwen3VLVideoProcessor(patch_size=ip.patch_size, temporal_patch_size=ip.temporal_patch_size,
                                 merge_size=ip.merge_size, size=dict(ip.size), image_mean=list(ip.image_mean),
                                 image_std=list(ip.image_std))


def prepare_video_request(prompt: list[int], video, model, model_dir: str | None = None,
                          processor_kwargs: dict | None = None, fps: float = 2.0,
                          images=None) -> tuple[list[int], MultiModalInputs]:
    """Video (frames ``[T, H, W, 3]``) of a Qwen3-VL request, optionally with images.  Qwen3-VL
    separates a video's temporal patch groups by timestamp text (``<t seconds> <vision_start>
    <video_pad> ... <vision_end>`` per group), so each group is one vision span with grid
    (1, h, w): the prompt must already hold those spans (the HF processor's layout; ``video_pad``
    repeated h w / merge^2 times per group).  Images and video spans are matched to the prompt in
    order of appearance.  Reference: Qwen3-VL video inputs
    (vllm_neuron/model/qwen3_vl/utils/vision_preprocessing.py)."""
    from ..models.qwen3_vl import mrope_positions

    vc = model.cfg.raw.get("vision_config") or {}
    vp = _video_processor(model_dir, vc, processor_kwargs)
    frames = np.asarray(video)
    out = vp(videos=[frames], return_tensors="pt", do_sample_frames=False,
             video_metadata=[{"fps": fps, "total_num_frames": int(frames.shape[0])}])
    vpix = out["pixel_values_videos"]
    t, h, w = (int(v) for v in out["video_grid_thw"][0].tolist())
    vgrids = [(1, h, w)] * t
    ipix, igrids = None, []
    if images is not None:
        if not isinstance(images, (list, tuple)):
            images = [images]
        o = _processor(model_dir, vc, processor_kwargs)(images=list(images), return_tensors="pt")
        ipix = o["pixel_values"]
        igrids = [tuple(int(v) for v in g) for g in o["image_grid_thw"].tolist()]
    m = model.spatial_merge
    img, vid = model.image_token_id, model.video_token_id
    # order the vision spans as they appear in the prompt
    grids, parts = [], []
    ii = vi = 0
    ioff = voff = 0
    i = 0
    ids = list(prompt)
    while i < len(ids):
        x = ids[i]
        if x == img or x == vid:
            gl = igrids if x == img else vgrids
            k = ii if x == img else vi
            if k >= len(gl):
                raise ValueError("more vision spans in the prompt than images / video groups")
            gt, gh, gw = gl[k]
            n = gt * gh * gw // (m * m)
            npatch = gt * gh * gw
            if x == img:
                parts.append(ipix[ioff:ioff + npatch])
                ioff += npatch
                ii += 1
            else:
                parts.append(vpix[voff:voff + npatch])
                voff += npatch
                vi += 1
            grids.append((gt, gh, gw))
            i += n
        else:
            i += 1
    if vi != len(vgrids) or ii != len(igrids):
        raise ValueError(f"prompt holds {vi} of {len(vgrids)} video groups and {ii} of {len(igrids)} images "
                         "(spans must be expanded: video_pad x h w / merge^2 per temporal group)")
    pos3, delta = mrope_positions(ids, {img, vid}, grids, m)
    rows = np.array([j for j, x in enumerate(ids) if x == img or x == vid], dtype=np.int64)
    mm = MultiModalInputs(pixels=torch.cat(parts), grids=grids, positions3=pos3, delta=delta, image_rows=rows)
    mm.row_of = {int(r): j for j, r in enumerate(rows)}
    return ids, mm


def prepare_image_request(prompt: list[int], images, model, model_dir: str | None = None,
                          processor_kwargs: dict | None = None) -> tuple[list[int], MultiModalInputs]:
    """Expand the image placeholders of ``prompt`` and build its MultiModalInputs."""
    from ..models.qwen3_vl import mrope_positions

    if not isinstance(images, (list, tuple)):
        images = [images]
    proc = _processor(model_dir, model.cfg.raw.get("vision_config") or {}, processor_kwargs)
    out = proc(images=list(images), return_tensors="pt")
    pixels = out["pixel_values"]
    grids = [tuple(int(v) for v in g) for g in out["image_grid_thw"].tolist()]
    m = model.spatial_merge
    counts = [t * h * w // (m * m) for t, h, w in grids]
    img = model.image_token_id
    n_ph = sum(1 for x in prompt if x == img)
    if n_ph == len(images):  # one placeholder per image: expand
        ids, k = [], 0
        for x in prompt:
            if x == img:
                ids.extend([img] * counts[k])
                k += 1
            else:
                ids.append(x)
    elif n_ph == sum(counts):
        ids = list(prompt)
    else:
        raise ValueError(f"prompt has {n_ph} image placeholders for {len(images)} images "
                         f"({sum(counts)} image tokens)")
    pos3, delta = mrope_positions(ids, img, grids, m)
    rows = np.array([i for i, x in enumerate(ids) if x == img], dtype=np.int64)
    mm = MultiModalInputs(pixels=pixels, grids=grids, positions3=pos3, delta=delta, image_rows=rows)
    mm.row_of = {int(r): j for j, r in enumerate(rows)}
    return ids, mm
