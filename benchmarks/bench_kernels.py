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
from vllm_neuron_b200.ops import attention as A  # noqa: E402
from vllm_neuron_b200.ops import linear as L  # noqa: E402
from vllm_neuron_b200.ops._ext import ext  # noqa: E402

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
            extra = {}
            if kind == "wide" and ext().gemm_2sm_enabled():
                # the single-SM kernel on the same shape (the CTA-pair kernel serves M >= 512)
                ext().gemm_2sm_set(False)
                t1 = timeit(fn)
                ext().gemm_2sm_set(True)
                extra = {"one_sm_ms": t1, "one_sm_tflops": flops / t1 / 1e9}
            bytes_ = (M * K + N * K) * 2 + M * N * 2
            rows.append({
                "op": f"gemm_{name}", "M": M, "N": N, "K": K, "kind": kind,
                "ms": t, "tflops": flops / t / 1e9, "gbs": bytes_ / t / 1e6,
                "cublas_ms": t_ref, "cublas_tflops": flops / t_ref / 1e9,
                "speedup_vs_cublas": t_ref / t, **extra,
            })
            print(json.dumps(rows[-1]), flush=True)
    return rows


def bench_gemms_decode_splits(tp: int):
    """Decode projections (64 and 16 tokens) under the split choices of the fp32-reduction
    kernel: the automatic pick, stream-K (-1) and fixed split-K factors, next to cuBLAS."""
    H, I, Hq, Hkv, D = 4096, 14336, 32, 8, 128
    shapes = {"qkv": ((Hq + 2 * Hkv) * D // tp, H), "o_proj": (H, Hq * D // tp),
              "gate_up": (2 * I // tp, H), "down": (H, I // tp)}
    rows = []
    for M in (64, 16):
        for name, (N, K) in shapes.items():
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
            acc = torch.zeros(M, N, device="cuda", dtype=torch.float32)
            r = {"op": f"decode_{name}", "M": M, "N": N, "K": K,
                 "cublas_us": timeit(lambda: torch.matmul(x, w.t())) * 1e3}
            for sp in (None, -1, 2, 3, 4, 6, 8):
                r[f"splits_{sp}_us"] = timeit(lambda: L.gemm_accumulate(x, w, acc, splits=sp)) * 1e3
            print(json.dumps(r), flush=True)
            rows.append(r)
    return rows


def bench_gemms_fp8(tp: int):
    """Static FP8 (W8A8) projections of the Llama-3-8B shapes next to the bf16 kernels: the time
    includes the activation quantization kernel; bytes count the fp8 weight."""
    H, I, Hq, Hkv, D = 4096, 14336, 32, 8, 128
    shapes = {"qkv": ((Hq + 2 * Hkv) * D // tp, H), "o_proj": (H, Hq * D // tp),
              "gate_up": (2 * I // tp, H), "down": (H, I // tp)}
    rows = []
    dev = "cuda"
    for M in (8192, 64):
        for name, (N, K) in shapes.items():
            x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
            w = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
            fw = L.FP8Weight.from_weight(w, in_scale=float(x.float().abs().max()) / 448)
            if M > L.SKINNY_MAX:
                out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                fn8 = lambda: L.gemm_out(x, fw, out)
                fn16 = lambda: L.gemm_out(x, w, out)
            else:
                acc = torch.zeros(M, N, device=dev, dtype=torch.float32)
                fn8 = lambda: L.gemm_accumulate(x, fw, acc)
                fn16 = lambda: L.gemm_accumulate(x, w, acc)
            t8, t16 = timeit(fn8), timeit(fn16)
            rows.append({"op": f"gemm_fp8_{name}", "M": M, "N": N, "K": K, "fp8_ms": t8, "bf16_ms": t16,
                         "fp8_tflops": 2.0 * M * N * K / t8 / 1e9, "fp8_weight_gbs": N * K / t8 / 1e6,
                         "speedup_vs_bf16": t16 / t8})
            print(json.dumps(rows[-1]), flush=True)
    return rows


def bench_gemms_fp8_block(tp: int):
    """128 x 128 block-FP8 weights (Llama-3-70B shapes per TP shard): W8A16 (weights widened to
    bf16 in shared memory) against W8A8 (1 x 128 fp8 activation blocks, per-k-block promotion),
    activation quantization included; bytes count the fp8 weight.  Also MXFP8 (e8m0 scale per 32
    elements, hardware block scaling) and the bf16-weight GEMM of the same shape."""
    H, I, Hq, Hkv, D = 8192, 28672, 64, 8, 128
    shapes = {"qkv": ((Hq + 2 * Hkv) * D // tp, H), "o_proj": (H, Hq * D // tp),
              "gate_up": (2 * I // tp, H), "down": (H, I // tp)}
    rows = []
    dev = "cuda"
    prev = L.fp8_block_activations()
    for M in (4096, 64, 16):
        for name, (N, K) in shapes.items():
            x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
            bw = L.BlockFP8Weight.from_weight(torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02)
            if M > L.SKINNY_MAX:
                out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                fn = lambda: L.gemm_out(x, bw, out)
            else:
                acc = torch.zeros(M, N, device=dev, dtype=torch.float32)
                fn = lambda: L.gemm_accumulate(x, bw, acc)
            t = {}
            for mode in ("bf16", "fp8"):
                L.set_fp8_block_activations(mode)
                t[mode] = timeit(fn)
            L.set_fp8_block_activations(prev)
            if M <= L.SKINNY_MAX:
                # the W8A8 kernel itself at every decode size (the op routes W8A8 up to 32 tokens)
                def w8a8_direct():
                    xq, xs = L.quantize_fp8_blocks(x)
                    tiles = -(-N // 128)
                    sp = L.pick_splits(N, K, L.num_sms(x.device), 128) if tiles < L.num_sms(x.device) else -1
                    ext().gemm_fp8_block(bw.q, xq, acc, L.skinny_bn(M), sp, bw.scales, xs)
                t["fp8"] = timeit(w8a8_direct)
            # MXFP8 (per-32 e8m0 scales) on the block-scaled MMA, activation quantization included,
            # and the bf16-weight GEMM of the same shape for context
            mw = L.MXFP8Weight.from_weight(bw.dequant_bf16_ref())
            wb = bw.dequant_bf16_ref()
            if M > L.SKINNY_MAX:
                t["mx8"] = timeit(lambda: L.gemm_out(x, mw, out))
                t["w16"] = timeit(lambda: L.gemm_out(x, wb, out))
            else:
                t["mx8"] = timeit(lambda: L.gemm_accumulate(x, mw, acc))
                t["w16"] = timeit(lambda: L.gemm_accumulate(x, wb, acc))
            rows.append({"op": f"gemm_fp8_block_{name}", "M": M, "N": N, "K": K,
                         "w8a16_ms": t["bf16"], "w8a8_ms": t["fp8"],
                         "w8a8_tflops": 2.0 * M * N * K / t["fp8"] / 1e9,
                         "w8a8_weight_gbs": N * K / t["fp8"] / 1e6, "speedup": t["bf16"] / t["fp8"],
                         "mx8_ms": t["mx8"], "mx8_tflops": 2.0 * M * N * K / t["mx8"] / 1e9,
                         "mx8_weight_gbs": N * K / t["mx8"] / 1e6, "bf16_weights_ms": t["w16"]})
            print(json.dumps(rows[-1]), flush=True)
    return rows


def bench_decode_attention(tp: int):
    Hq, Hkv, D, bs = 32 // tp, max(1, 8 // tp), 128, 16
    rows = []
    for B, ctx, kvdt in ((64, 1152, "bf16"), (64, 4096, "bf16"), (16, 8192, "bf16"),
                         (64, 1152, "fp8"), (64, 4096, "fp8")):
        nblk = (ctx + bs - 1) // bs
        nb = B * nblk + 1
        kc = torch.randn(nb, Hkv, bs, D, device="cuda", dtype=torch.bfloat16)
        vc = torch.randn_like(kc)
        if kvdt == "fp8":
            kc, vc = kc.to(torch.float8_e4m3fn), vc.to(torch.float8_e4m3fn)
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
        kv_bytes = 2 * B * ctx * Hkv * D * kc.element_size()
        rows.append({"op": "decode_attention", "kv": kvdt, "B": B, "ctx": ctx, "Hq": Hq, "Hkv": Hkv,
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
        out = torch.empty_like(q)
        flops = 4.0 * B * S * S / 2 * Hq * D
        # 64-row items run the mma.sync kernel, 128-row items the tcgen05 (TMEM) kernel
        for pr in sorted({A.PREFILL_ROWS, A.prefill_rows(D, kc.dtype, bs, Hq // Hkv)}):
            w = ops.build_work(np.full(B, S), sl.cpu().numpy(), Hq // Hkv, Hkv, prefill_rows=pr)
            work = torch.from_numpy(w.work).cuda()
            fn = lambda: ops.paged_attention(q, kc, vc, bt, sl, qs, work, False, 1, 1 / math.sqrt(D), out=out,
                                             prefill_rows=pr)
            t = timeit(fn)
            rows.append({"op": "prefill_attention", "rows": pr, "B": B, "S": S, "Hq": Hq, "ms": t,
                         "tflops": flops / t / 1e9})
            print(json.dumps(rows[-1]), flush=True)
    return rows


def bench_moe(tp: int):
    """GPT-OSS-20B expert block (32 experts top-4, hidden 2880, FFN 2880) at decode batch sizes:
    bf16 grouped tcgen05 GEMMs, the MXFP4 mma.sync decode kernel and the MXFP4 tcgen05 GEMM
    (swapped grouped mode up to 64 tokens, W4A16 grouped above) on the same routing and weights,
    each block replayed from a CUDA graph.  The weight bandwidth counts only the active experts'
    weight bytes (router, routing and combine time included in the denominator)."""
    from vllm_neuron_b200.models.gpt_oss import _quant_experts, dequant_mxfp4
    from vllm_neuron_b200.ops import moe as M

    E, k, H, I = 32, 4, 2880, 2880 // tp
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    gu_b, gu_s = _quant_experts(torch.randn(E, 2 * I, H, device=dev, generator=g) * H ** -0.5)
    dn_b, dn_s = _quant_experts(torch.randn(E, H, I, device=dev, generator=g) * I ** -0.5)
    w_gu, w_dn = dequant_mxfp4(gu_b, gu_s), dequant_mxfp4(dn_b, dn_s)
    fp4_gu, fp4_dn = M.pack_mxfp4(gu_b, gu_s), M.pack_mxfp4(dn_b, dn_s)
    mx_gu, mx_dn = L.MXFP4Weight.from_blocks(gu_b, gu_s), L.MXFP4Weight.from_blocks(dn_b, dn_s)
    rw = (torch.randn(E, H, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    ws = M.MoEWorkspace.create(128, k, E, E, H, I, dev)
    rows = []
    for T in (1, 8, 32, 64, 128):
        x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)

        def graph(fp4: bool, tc: bool = False):
            kw = dict(fp4_gu=fp4_gu, fp4_down=fp4_dn, fp4_max_tokens=1 << 20) if fp4 else {}
            wg, wd = (mx_gu, mx_dn) if tc else (w_gu, w_dn)
            run = lambda: M.moe_block(x, rw, wg, wd, k, M.ROUTE_TOPK_SOFTMAX, act=M.ACT_GPTOSS, ws=ws, **kw)
            run()  # compile-time setup (shared-memory opt-in) outside the capture
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                run()
            return gr.replay

        # decode replays the block from a CUDA graph; time it the same way (no host gaps)
        t_bf16 = timeit(graph(False))
        t_fp4 = timeit(graph(True))
        t_tc = timeit(graph(False, tc=True))
        active = int(torch.unique(ws.ids[:T]).numel())
        fp4_bytes = active * (fp4_gu[0].numel() + fp4_dn[0].numel())
        bf16_bytes = active * (w_gu[0].numel() + w_dn[0].numel()) * 2
        r = {"kernel": "moe_block_gptoss", "T": T, "tp": tp, "active_experts": active,
             "bf16_us": t_bf16 * 1e3, "fp4_mma_sync_us": t_fp4 * 1e3, "fp4_tcgen05_us": t_tc * 1e3,
             "bf16_weight_GBs": bf16_bytes / (t_bf16 * 1e-3) / 1e9,
             "fp4_mma_sync_weight_GBs": fp4_bytes / (t_fp4 * 1e-3) / 1e9,
             "fp4_tcgen05_weight_GBs": fp4_bytes / (t_tc * 1e-3) / 1e9}
        print(json.dumps(r), flush=True)
        rows.append(r)
    return rows


def bench_deltanet(tp: int):
    """Gated DeltaNet layer of the Qwen3.6-A3B shape (16 key / 32 value heads x 128) per TP
    shard: prefill of 8 x 1024 tokens (one 8192-token chunk) and a 64-sequence decode step.
    Time covers the q/k normalisation pass, the recurrence (token by token, or the chunked WY
    form for the prefill) and the gated RMSNorm."""
    from vllm_neuron_b200.ops import deltanet as DN

    Hk, Hv, d = 16 // tp, 32 // tp, 128
    dev = "cuda"
    rows = []
    for name, q_lens, ctx, mode in (("prefill_8x1024", [1024] * 8, [0] * 8, "recurrent"),
                                    ("prefill_8x1024_chunked", [1024] * 8, [0] * 8, "chunked"),
                                    ("prefill_2x4096_chunked", [4096] * 2, [0] * 2, "chunked"),
                                    ("decode_b64", [1] * 64, [2048] * 64, "recurrent")):
        B = len(q_lens)
        qs = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32, device=dev)
        sl = torch.tensor([a + b for a, b in zip(q_lens, ctx)], dtype=torch.int32, device=dev)
        slots = torch.arange(B, dtype=torch.int32, device=dev)
        T = sum(q_lens)
        qkv = torch.randn(T, 2 * Hk * d + Hv * d, device=dev).to(torch.bfloat16)
        zab = torch.randn(T, Hv * d + 2 * Hv, device=dev).to(torch.bfloat16)
        z, b, a = zab[:, :Hv * d], zab[:, Hv * d:Hv * d + Hv], zab[:, Hv * d + Hv:]
        A_log = torch.rand(Hv, device=dev).add(0.5).log()
        dt_bias = torch.zeros(Hv, device=dev)
        nw = torch.ones(d, device=dev, dtype=torch.bfloat16)
        state = torch.zeros(B, Hv, d, d, device=dev)
        out = torch.empty(T, Hv * d, device=dev, dtype=torch.bfloat16)
        ms = timeit(lambda: DN.gated_delta_rule(qkv, z, a, b, A_log, dt_bias, nw, 1e-6, qs, sl, slots,
                                                state, out, Hk, Hv, mode=mode))
        r = {"op": "gated_delta_rule", "case": name, "mode": mode, "tp": tp, "T": T, "ms": ms,
             "us_per_token_step": ms * 1e3 / max(q_lens)}
        print(json.dumps(r), flush=True)
        rows.append(r)
    return rows


def profile_case(name: str):
    """Run one kernel three times on one shape without timing (the target of an ncu capture:
    ``ncu -k regex:<kernel> -s 1 -c 1 python benchmarks/bench_kernels.py --profile-case NAME``).

    fmha       tcgen05 prefill attention, 2 x 4096 tokens, Llama-3-8B heads (fmha_prefill_kernel)
    gemm2sm    gate/up + SwiGLU projection, M = 8192, N = 28672, K = 4096 (gemm2sm_kernel)
    gemm_dec   decode gate/up projection, M = 64, stream-K fp32 reduction (gemm_bf16_kernel)
    mx8_dec    MXFP8 decode gate/up, Llama-3-70B TP2 shard (N = 28672, K = 8192), M = 64
    mx8_pre    MXFP8 prefill gate/up, same shard, M = 4096 (bf16 store)
    """
    if name == "fmha":
        Hq, Hkv, D, bs, B, S = 32, 8, 128, 16, 2, 4096
        nblk = S // bs
        nb = B * nblk + 1
        kc = torch.randn(nb, Hkv, bs, D, device="cuda", dtype=torch.bfloat16)
        vc = torch.randn_like(kc)
        bt = (torch.randperm(nb - 1, device="cuda")[: B * nblk] + 1).view(B, nblk).to(torch.int32)
        sl = torch.full((B,), S, dtype=torch.int32, device="cuda")
        qs = torch.arange(0, (B + 1) * S, S, dtype=torch.int32, device="cuda")
        q = torch.randn(B * S, Hq, D, device="cuda", dtype=torch.bfloat16)
        pr = A.prefill_rows(D, kc.dtype, bs, Hq // Hkv)
        w = ops.build_work(np.full(B, S), sl.cpu().numpy(), Hq // Hkv, Hkv, prefill_rows=pr)
        work = torch.from_numpy(w.work).cuda()
        out = torch.empty_like(q)
        fn = lambda: ops.paged_attention(q, kc, vc, bt, sl, qs, work, False, 1, 1 / math.sqrt(D), out=out,
                                         prefill_rows=pr)
    elif name == "gemm2sm":
        x = torch.randn(8192, 4096, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(28672, 4096, device="cuda", dtype=torch.bfloat16) * 0.02
        out = torch.empty(8192, 14336, device="cuda", dtype=torch.bfloat16)
        fn = lambda: L.gemm_silu(x, w, out=out)
    elif name == "gemm_dec":
        x = torch.randn(64, 4096, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(28672, 4096, device="cuda", dtype=torch.bfloat16) * 0.02
        acc = torch.zeros(64, 28672, device="cuda", dtype=torch.float32)
        fn = lambda: L.gemm_accumulate(x, w, acc)
    elif name in ("mx8_dec", "mx8_pre"):
        M = 64 if name == "mx8_dec" else 4096
        x = torch.randn(M, 8192, device="cuda", dtype=torch.bfloat16)
        mw = L.MXFP8Weight.from_weight(torch.randn(28672, 8192, device="cuda", dtype=torch.bfloat16) * 0.02)
        if M <= L.SKINNY_MAX:
            acc = torch.zeros(M, 28672, device="cuda", dtype=torch.float32)
            fn = lambda: L.gemm_accumulate(x, mw, acc)
        else:
            out = torch.empty(M, 28672, device="cuda", dtype=torch.bfloat16)
            fn = lambda: L.gemm_out(x, mw, out)
    else:
        raise SystemExit(f"unknown profile case {name}")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    print("profile case", name, "done", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile-case", type=str, default=None, help="fmha | gemm2sm | gemm_dec | mx8_dec | mx8_pre (see profile_case)")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--json", type=str, default=None)
    ap.add_argument("--only", type=str, default="gemm,decode,prefill,moe,deltanet")
    a = ap.parse_args()
    torch.manual_seed(0)
    if a.profile_case:
        return profile_case(a.profile_case)
    rows = []
    only = a.only.split(",")
    if "gemm" in only:
        rows += bench_gemms(a.tp)
    if "gemmdec" in only:
        rows += bench_gemms_decode_splits(a.tp)
    if "fp8gemm" in only:
        rows += bench_gemms_fp8(a.tp)
    if "fp8block" in only:
        rows += bench_gemms_fp8_block(a.tp)
    if "decode" in only:
        rows += bench_decode_attention(a.tp)
    if "prefill" in only:
        rows += bench_prefill_attention(a.tp)
    if "moe" in only:
        rows += bench_moe(a.tp)
    if "deltanet" in only:
        rows += bench_deltanet(a.tp)
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
