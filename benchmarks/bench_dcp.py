"""Decode attention under decode context parallelism, one GPU: the time of one DCP rank's
partial attention over its 1/d share of every sequence (Q gathered: d x the local query heads)
plus the LSE merge of d partials, against plain TP decode attention over the whole context.
Communication (the Q all-gather and the partial all-to-all) is not included.

    python benchmarks/bench_dcp.py [--batch 64] [--ctx 8192] [--dcp 2]
"""
import argparse
import json
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from vllm_neuron_b200 import ops  # noqa: E402


def _time(fn, iters=20, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--dcp", type=int, default=2)
    ap.add_argument("--q-heads", type=int, default=4, help="query heads per rank (one KV head)")
    a = ap.parse_args()
    dev, D, bs, B, d = "cuda", 128, 16, a.batch, a.dcp
    Hl = a.q_heads
    ctx = a.ctx
    nblk = ctx // bs
    scale = D ** -0.5
    q_start = torch.arange(B + 1, dtype=torch.int32, device=dev)
    bt = torch.arange(1, 1 + B * nblk, dtype=torch.int32, device=dev).view(B, nblk)
    k = torch.randn(1 + B * nblk, 1, bs, D, device=dev).to(torch.bfloat16)
    v = torch.randn_like(k)
    # plain TP: the local heads over the whole context
    sl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, Hl, D, device=dev).to(torch.bfloat16)
    w = ops.build_work(np.ones(B), np.full(B, ctx), Hl, 1, 148, head_dim=D)
    work = torch.from_numpy(w.work).to(dev)
    out = torch.empty_like(q)
    t_full = _time(lambda: ops.paged_attention(q, k, v, bt, sl, q_start, work, True, w.num_splits,
                                               scale, out=out))
    # DCP rank 0: d x the heads (gathered Q) over its 1/d of the tokens, then the merge
    local = ops.dcp_local_count(ctx, bs, d, 0)
    lsl = torch.full((B,), local, dtype=torch.int32, device=dev)
    qg = torch.randn(B, Hl * d, D, device=dev).to(torch.bfloat16)
    wd = ops.build_work(np.ones(B), np.full(B, local), Hl * d, 1, 148, head_dim=D)
    workd = torch.from_numpy(wd.work).to(dev)
    ns = wd.num_splits
    po = torch.empty(ns, B, Hl * d, D, device=dev)
    pl = torch.empty(ns, B, Hl * d, device=dev)
    t_part = _time(lambda: ops.paged_attention_partial(qg, k, v, bt, lsl, q_start, workd, True, ns,
                                                       scale, po, pl, dcp_seq_lens=sl, dcp_size=d,
                                                       dcp_rank=0))
    ro = torch.randn(d * ns, B, Hl, D, device=dev)
    rl = torch.randn(d * ns, B, Hl, device=dev)
    t_merge = _time(lambda: ops.attn_combine(ro, rl, out))
    kv_bytes_full = 2 * B * ctx * D * 2
    print(json.dumps({"batch": B, "ctx": ctx, "dcp": d, "q_heads_local": Hl,
                      "tp_attn_ms": round(t_full, 4), "tp_splits": w.num_splits,
                      "dcp_partial_ms": round(t_part, 4), "dcp_splits": ns,
                      "dcp_merge_ms": round(t_merge, 4),
                      "tp_kv_gbs": round(kv_bytes_full / t_full / 1e6, 1),
                      "dcp_kv_gbs": round(kv_bytes_full / d / t_part / 1e6, 1),
                      "kv_tokens_per_rank": {"tp": ctx, "dcp": local}}))


if __name__ == "__main__":
    main()
