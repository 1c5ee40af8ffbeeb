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
