"""The JSON record written beside each captured step: what ran (step index, ranks, decode or
prefill, split factor, work items), on what (model architecture, dtype, KV cache shape) and for
whom (request ids, the positions each computed, whether it sampled).  Reference:
vllm_neuron/snapshot/meta.py (write_call_meta)."""
from __future__ import annotations

import json
import os
import time


def write_step_meta(path: str, *, step: int, rank: int, world: int, decode: bool, num_splits: int,
                    work_len: int, layout: dict, requests: list[dict], model: dict, fmt: str) -> str:
    rec = {"version": 1, "time": time.time(), "step": step, "rank": rank, "world": world,
           "decode": bool(decode), "num_splits": int(num_splits), "work_len": int(work_len),
           "layout": layout, "requests": requests, "model": model, "format": fmt}
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        json.dump(rec, f, indent=1)
    os.replace(tmp, path)
    return path


def read_step_meta(path: str) -> dict:
    with open(path) as f:
        return json.load(f)
