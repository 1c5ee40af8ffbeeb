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


def load_checkpoint_into(model, path: str) -> dict:
    t0 = time.perf_counter()
    ck = SafetensorsCheckpoint(path)
    warm = ck.warm_page_cache(model.tp.rank, model.tp.world)
    model.load_hf_state_dict(ck.get, ck.names())
    warm.join(timeout=0)
    if torch.cuda.is_available() and model.device.type == "cuda":
        torch.cuda.synchronize(model.device)
    return {"seconds": time.perf_counter() - t0, "bytes": ck.bytes_read}
