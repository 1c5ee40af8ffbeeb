"""Capture of selected steps' device inputs.

The model runner packs every step's inputs (token ids, positions, slots, block tables, sequence
lengths, attention work items, sampling parameters) into one pinned int32 buffer with a layout of
offsets; :class:`SnapshotCapturer` saves that buffer and its layout -- exactly what the device
received -- plus a metadata record, for the steps the configuration selects.  Files per step:
``rank<r>_step<nnnnnn>.pt`` (or ``.npy`` + ``.layout.json``) and ``...meta.json``.
Reference: vllm_neuron/snapshot/capture.py (SnapshotCapturer.pre_execute).
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch

from .config import SnapshotConfig
from .meta import write_step_meta


class SnapshotCapturer:
    def __init__(self, config: SnapshotConfig, rank: int = 0, world: int = 1):
        self.cfg = config
        self.rank, self.world = rank, world
        self.step = 0          # steps seen by this runner
        self.captured = 0
        self.enabled = config.active and config.rank_enabled(rank)
        if self.enabled:
            os.makedirs(config.directory, exist_ok=True)

    def pre_execute(self, out, lay, buffer: torch.Tensor, decode: bool, splits: int, work_len: int,
                    model, prefill_rows: int = 64) -> str | None:
        """Called before a step runs: saves it when selected; returns the metadata path."""
        step = self.step
        self.step += 1
        if not self.enabled or self.captured >= self.cfg.max_steps:
            return None
        ranges = [(s.start, s.start + s.num_tokens) for s in out.scheduled]
        rids = [s.req.request_id for s in out.scheduled]
        if not self.cfg.selector.matches(step, ranges, rids):
            return None
        base = os.path.join(self.cfg.directory, f"rank{self.rank}_step{step:06d}")
        layout = dict(T=lay.T, B=lay.B, S=lay.S, W=lay.W, nblk=lay.nblk, total=lay.total,
                      offsets={k: list(v) for k, v in lay.off.items()})
        reqs = [{"request_id": s.req.request_id, "start": s.start, "num_tokens": s.num_tokens,
                 "samples": bool(s.samples), "spec": list(s.spec),
                 "prompt_len": len(s.req.prompt_token_ids)} for s in out.scheduled]
        host = buffer[:lay.total].clone()
        if self.cfg.fmt == "pt":
            torch.save({"step": step, "layout": layout, "buffer": host, "decode": decode,
                        "num_splits": splits, "work_len": work_len, "requests": reqs,
                        "prefill_rows": prefill_rows}, base + ".pt")
        else:
            np.save(base + ".npy", host.numpy())
            with open(base + ".layout.json", "w") as f:
                json.dump({"layout": layout, "decode": decode, "num_splits": splits, "work_len": work_len,
                           "prefill_rows": prefill_rows}, f)
        m = model
        minfo = {"class": type(m).__name__, "layers": len(getattr(m, "layers", [])),
                 "hidden": getattr(m, "H", None), "head_dim": getattr(m, "D", None),
                 "kv_dtype": str(getattr(m, "kv_dtype", "")), "dtype": str(getattr(m, "dtype", ""))}
        self.captured += 1
        return write_step_meta(base + ".meta.json", step=step, rank=self.rank, world=self.world,
                               decode=decode, num_splits=splits, work_len=work_len, layout=layout,
                               requests=reqs, model=minfo, fmt=self.cfg.fmt)
