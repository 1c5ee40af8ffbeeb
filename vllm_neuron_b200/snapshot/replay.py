"""Replay of a captured step: the saved int32 input buffer is copied to the runner's device
buffer and unpacked with the saved layout, and the model runs the step again, returning the
logits of its sampling rows.  A prefill step of requests without cached context depends on
nothing else and reproduces its logits; decode and chunked-prefill steps read the KV cache, so
they match only against the cache state they originally ran with."""
from __future__ import annotations

import json
import os

import numpy as np
import torch


class _Lay:
    def __init__(self, d: dict):
        self.T, self.B, self.S, self.W, self.nblk = d["T"], d["B"], d["S"], d["W"], d["nblk"]
        self.total = d["total"]
        self.off = {k: tuple(v) for k, v in d["offsets"].items()}


def load_snapshot(path: str) -> dict:
    """``rank<r>_step<n>.pt`` (or the ``.npy`` with its ``.layout.json``) -> dict with ``buffer``
    (int32 tensor), ``layout``, ``decode``, ``num_splits``, ``work_len``."""
    if path.endswith(".npy"):
        with open(path[:-4] + ".layout.json") as f:
            d = json.load(f)
        d["buffer"] = torch.from_numpy(np.load(path))
        return d
    return torch.load(path)


@torch.no_grad()
def replay_logits(runner, snap: dict) -> torch.Tensor:
    """Run the captured step on ``runner`` (same model and configuration) and return the logits
    of its sampling rows ``[S, V]``."""
    lay = _Lay(snap["layout"])
    buf = snap["buffer"]
    dev = runner.dev_buf[:lay.total]
    dev.copy_(buf.to(dev.device))
    fb, _ = runner._views(dev, lay, lay.B, lay.S, snap["work_len"], snap["decode"], snap["num_splits"])
    fb.work = fb.work[:snap["work_len"]]
    fb.prefill_rows = snap.get("prefill_rows", fb.prefill_rows)
    logits = runner.model.forward(fb).clone()
    if runner.is_cuda:
        torch.cuda.synchronize(runner.device)
    return logits


def list_snapshots(directory: str, rank: int = 0) -> list[str]:
    return sorted(os.path.join(directory, f) for f in os.listdir(directory)
                  if f.startswith(f"rank{rank}_step") and (f.endswith(".pt") or f.endswith(".npy")))
