"""Safetensors checkpoint access with a background page-cache warmer.

``SafetensorsCheckpoint`` indexes every tensor of a local HF directory
(``model.safetensors.index.json`` or ``*.safetensors``) and reads tensors lazily through
memory-mapped files.  ``load_checkpoint_into(model, path)`` hands the tensor getter to the
model's loader (which shards/fuses per rank).  While the main thread transforms tensors, a
background thread reads ahead the remaining files so their pages are resident (the
pipelined loading of the reference: vllm_neuron/utils/checkpoints.py:26-681).
"""
from __future__ import annotations

import glob
import json
import os
import threading
import time

import torch


class SafetensorsCheckpoint:
    def __init__(self, path: str):
        from safetensors import safe_open  # noqa: F401  (dependency check)

        self.path = path
        idx = os.path.join(path, "model.safetensors.index.json")
        self.name_to_file: dict[str, str] = {}
        if os.path.exists(idx):
            with open(idx) as f:
                wm = json.load(f)["weight_map"]
            self.name_to_file = {k: os.path.join(path, v) for k, v in wm.items()}
        else:
            from safetensors import safe_open

            for fn in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
                with safe_open(fn, framework="pt") as f:
                    for k in f.keys():
                        self.name_to_file[k] = fn
        if not self.name_to_file:
            raise FileNotFoundError(f"no safetensors weights under {path}")
        self._handles = {}
        self._lock = threading.Lock()
        self.bytes_read = 0

    def names(self) -> set[str]:
        return set(self.name_to_file)

    def _handle(self, fn):
        from safetensors import safe_open

        with self._lock:
            h = self._handles.get(fn)
            if h is None:
                h = safe_open(fn, framework="pt")
                self._handles[fn] = h
            return h

    def get(self, name: str) -> torch.Tensor:
        fn = self.name_to_file.get(name)
        if fn is None:
            raise KeyError(f"tensor {name!r} not in checkpoint {self.path}")
        t = self._handle(fn).get_tensor(name)
        self.bytes_read += t.numel() * t.element_size()
        return t

    def warm_page_cache(self, rank: int = 0, world: int = 1) -> threading.Thread:
        """Read this rank's share of the files in the background (sequential reads)."""
        files = sorted(set(self.name_to_file.values()))[rank::world]

        def run():
            for fn in files:
                try:
                    with open(fn, "rb") as f:
                        while f.read(64 << 20):
                            pass
                except OSError:
                    pass

        th = threading.Thread(target=run, daemon=True)
        th.start()
        return th


def dequant_block_fp8(w: torch.Tensor, scale_inv: torch.Tensor, block: tuple[int, int] = (128, 128),
                      dtype=torch.bfloat16) -> torch.Tensor:
    """Block-scaled fp8 (e4m3) weight ``[N, K]`` with per-block scales ``[ceil(N/bn), ceil(K/bk)]``
    -> ``dtype`` (``w * scale`` per block)."""
    bn, bk = block
    N, K = w.shape[-2], w.shape[-1]
    s = scale_inv.float().repeat_interleave(bn, -2)[..., :N, :].repeat_interleave(bk, -1)[..., :K]
    return (w.float() * s).to(dtype)


def quant_block_fp8(w: torch.Tensor, block: tuple[int, int] = (128, 128)) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of :func:`dequant_block_fp8` (amax / 448 per block); builds fp8 checkpoints."""
    bn, bk = block
    N, K = w.shape
    nb, kb = -(-N // bn), -(-K // bk)
    pad = torch.zeros(nb * bn, kb * bk, dtype=torch.float32)
    pad[:N, :K] = w.float()
    blocks = pad.view(nb, bn, kb, bk)
    scale = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12) / 448.0
    q = (blocks / scale[:, None, :, None]).view(nb * bn, kb * bk)[:N, :K].to(torch.float8_e4m3fn)
    return q, scale


def fp8_aware_getter(get, names: set[str], block: tuple[int, int] | None):
    """Wrap ``get`` so that fp8 weights with a ``*_scale_inv`` (block-scaled, the ModelOpt /
    DeepSeek / Qwen FP8 layout) are returned dequantized to bf16 (reference: block-FP8 and
    static FP8 checkpoint handling, vllm_neuron/model/llama3/quantization.py:39-310)."""
    blk = tuple(block) if block else (128, 128)

    def g(name: str) -> torch.Tensor:
        t = get(name)
        if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
            si = name + "_scale_inv"
            if si in names:
                return dequant_block_fp8(t, get(si), blk, torch.float32)
            sc = name.replace(".weight", ".weight_scale")
            if sc in names:
                s = get(sc)
                if s.dtype == torch.uint8 and s.dim() == t.dim() and s.shape[-1] * 32 == t.shape[-1]:
                    # MXFP8 (LLM-Compressor): one e8m0 scale per 32 elements, exact in bf16
                    g.mxfp8 = True
                    e = s.to(torch.int32) - 127
                    return (t.float().unflatten(-1, (-1, 32)) * torch.exp2(e.float())[..., None]).flatten(-2)
                return t.float() * s.float()  # per-tensor static scale
            return t.float()
        return t

    g.mxfp8 = False  # set once an MXFP8 weight was read
    return g


def load_checkpoint_into(model, path: str) -> dict:
    t0 = time.perf_counter()
    ck = SafetensorsCheckpoint(path)
    warm = ck.warm_page_cache(model.tp.rank, model.tp.world)
    names = ck.names()
    getter = fp8_aware_getter(ck.get, names, getattr(model.cfg, "weight_block_size", None))
    model.load_hf_state_dict(getter, names)
    warm.join(timeout=0)
    if torch.cuda.is_available() and model.device.type == "cuda":
        torch.cuda.synchronize(model.device)
    return {"seconds": time.perf_counter() - t0, "bytes": ck.bytes_read, "mxfp8": getter.mxfp8}
