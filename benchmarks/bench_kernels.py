"""Kernel microbenchmarks on one B200: the framework's sm_100a kernels next to the library
baseline (cuBLAS through torch.matmul) on the Llama-3-8B projection shapes, and decode
attention bandwidth.  Device-timed with CUDA events after warm-up; L2 is flushed (a 256 MiB
write) before every timed launch.

    python benchmarks/bench_kernels.py [--tp 1] [--json out.json]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from vllm_neuron_b200 import ops  # noqa: E402
from vllm_neuron_b200.ops import linear as L  # noqa: E402

_FLUSH = None


def flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.fill_(1)


def timeit(fn, iters=20, warmup=5, flush=True):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush_l2()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return float(np.median(times))


def bench_gemms(tp: int):
    H, I, Hq, Hkv, D = 4096, 14336, 32, 8, 128
    shapes = {
        "qkv": ((Hq + 2 * Hkv) * D // tp, H),
        "o_proj": (H, Hq * D // tp),
        "gate_up": (2 * I // tp, H),
        "down": (H, I // tp),
    }
    rows = []
    dev = "cuda"
    for M in (8192, 2048, 64, 16):
        for name, (N, K) in shapes.items():
            x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
            w = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
            flops = 2.0 * M * N * K
            t_ref = timeit(lambda: torch.matmul(x, w.t()))
            if M > L.SKINNY_MAX:
                if name == "gate_up":
                    fn = lambda: L.gemm_silu(x, w)
                else:
                    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                    fn = lambda: L.gemm_out(x, w, out)
                kind = "wide"
            else:
                acc = torch.zeros(M, N, device=dev, dtype=torch.float32)
                fn = lambda: L.gemm_accumulate(x, w, acc)
                kind = "splitk_f32"
            t = timeit(fn)
            bytes_ = (M * K + N * K) * 2 + M * N * 2
            rows.append({
                "op": f"gemm_{name}", "M": M, "N": N, "K": K, "kind": kind,
                "ms": t, "tflops": flops / t / 1e9, "gbs": bytes_ / t / 1e6,
                "cublas_ms": t_ref, "cublas_tflops": flops / t_ref / 1e9,
                "speedup_vs_cublas": t_ref / t,
            })
            print(json.dumps(rows[-1]), flush=True)
    return rows


def bench_decode_attention(tp: int):
    Hq, Hkv, D, bs = 32 // tp, max(1, 8 // tp), 128, 16
    rows = []
    for B, ctx in ((64, 1152), (64, 4096), (16, 8192)):
        nblk = (ctx + bs - 1) // bs
        nb = B * nblk + 1
        kc = torch.randn(nb, Hkv, bs, D, device="cuda", dtype=torch.bfloat16)
        vc = torch.randn_like(kc)
        bt = (torch.randperm(nb - 1, device="cuda")[: B * nblk] + 1).view(B, nblk).to(torch.int32)
        sl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
        qs = torch.arange(B + 1, dtype=torch.int32, device="cuda")
        q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
        w = ops.build_work(np.ones(B, dtype=np.int64), sl.cpu().numpy(), Hq // Hkv, Hkv)
        work = torch.from_numpy(w.work).cuda()
        out = torch.empty_like(q)
        part_o = torch.empty(w.num_splits, B, Hq, D, device="cuda")
        part_l = torch.empty(w.num_splits, B, Hq, device="cuda")
        fn = lambda: ops.paged_attention(q, kc, vc, bt, sl, qs, work, True, w.num_splits,
                                         1 / math.sqrt(D), out=out, part_o=part_o, part_lse=part_l)
        t = timeit(fn)
        kv_bytes = 2 * B * ctx * Hkv * D * 2
        rows.append({"op": "decode_attention", "B": B, "ctx": ctx, "Hq": Hq, "Hkv": Hkv,
                     "splits": w.num_splits, "ms": t, "gbs": kv_bytes / t / 1e6})
        print(json.dumps(rows[-1]), flush=True)
    return rows


def bench_prefill_attention(tp: int):
    Hq, Hkv, D, bs = 32 // tp, max(1, 8 // tp), 128, 16
    rows = []
    for B, S in ((8, 1024), (2, 4096)):
        nblk = (S + bs - 1) // bs
        nb = B * nblk + 1
        kc = torch.randn(nb, Hkv, bs, D, device="cuda", dtype=torch.bfloat16)
        vc = torch.randn_like(kc)
        bt = (torch.randperm(nb - 1, device="cuda")[: B * nblk] + 1).view(B, nblk).to(torch.int32)
        sl = torch.full((B,), S, dtype=torch.int32, device="cuda")
        qs = torch.arange(0, (B + 1) * S, S, dtype=torch.int32, device="cuda")
        q = torch.randn(B * S, Hq, D, device="cuda", dtype=torch.bfloat16)
        w = ops.build_work(np.full(B, S), sl.cpu().numpy(), Hq // Hkv, Hkv)
        work = torch.from_numpy(w.work).cuda()
        out = torch.empty_like(q)
        fn = lambda: ops.paged_attention(q, kc, vc, bt, sl, qs, work, False, 1, 1 / math.sqrt(D), out=out)
        t = timeit(fn)
        flops = 4.0 * B * S * S / 2 * Hq * D
        rows.append({"op": "prefill_attention", "B": B, "S": S, "Hq": Hq, "ms": t,
                     "tflops": flops / t / 1e9})
        print(json.dumps(rows[-1]), flush=True)
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--json", type=str, default=None)
    ap.add_argument("--only", type=str, default="gemm,decode,prefill")
    a = ap.parse_args()
    torch.manual_seed(0)
    rows = []
    only = a.only.split(",")
    if "gemm" in only:
        rows += bench_gemms(a.tp)
    if "decode" in only:
        rows += bench_decode_attention(a.tp)
    if "prefill" in only:
        rows += bench_prefill_attention(a.tp)
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
