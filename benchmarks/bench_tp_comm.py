"""Decode all-reduce benchmark: the fused all-reduce + residual + RMSNorm kernel against NCCL.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_tp_comm.py [--hidden 4096]

For each row count T it checks, on the first call, that the fused kernel (sentinel-polled
form and the per-row-flag form) gives the same residual and normalized rows as NCCL all-reduce +
add_rmsnorm (and that every rank holds identical rows), then times each path as a CUDA graph
of ``--calls`` back-to-back calls (CUDA events, after warm-up replays; max over ranks).

NVLink roofline per call: the bytes each rank must send for an all-reduce of the bf16 rows,
``2 (W - 1) / W * T * H * 2`` (reduce-scatter + all-gather), at the measured peer copy rate
(770 GB/s per direction); the one-shot fused kernel sends ``(W - 1) * T * H * 2``.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

LINK_GBS = 770.0  # measured NVLink peer copy per direction per GPU on this pool


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--rows", default="1,8,32,64,128")
    ap.add_argument("--calls", type=int, default=64)
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args()

    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops._ext import ext
    from vllm_neuron_b200.parallel import state as ps
    from vllm_neuron_b200.parallel.comm import GroupComm
    from vllm_neuron_b200.parallel.fused import TPFusedComm

    rank, world = ps.init_distributed(timeout_s=300)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tp = GroupComm(dist.group.WORLD, list(range(world)))
    cpu = dist.new_group(backend="gloo")
    H = args.hidden
    rows = [int(r) for r in args.rows.split(",")]
    Tmax = max(rows)
    comms = [TPFusedComm(tp, H, Tmax, dev, cpu, algo=a) for a in (0, 1)]  # one object per form
    w = (1.0 + 0.1 * torch.randn(H, device=dev, generator=torch.Generator(device=dev).manual_seed(3))
         ).to(torch.bfloat16)
    eps = 1e-5
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    acc = torch.zeros(Tmax, H, dtype=torch.float32, device=dev)
    res0 = torch.randn(Tmax, H, device=dev, generator=torch.Generator(device=dev).manual_seed(7)).to(torch.bfloat16)
    res = res0.clone()
    out = torch.empty(Tmax, H, dtype=torch.bfloat16, device=dev)
    results = []

    def timed(fn):
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            for _ in range(3):
                fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=s):
            for _ in range(args.calls):
                fn()
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (args.reps * args.calls)
        t = torch.tensor([us], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del gr
        return float(t.item())

    for T in rows:
        part = torch.randn(T, H, device=dev, generator=g) * 0.5
        # reference: NCCL all-reduce of the bf16-rounded partials (fp32 sum in rank order)
        allp = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(allp, part.to(torch.bfloat16).float())
        s = torch.zeros_like(part)
        for p_ in allp:
            s += p_
        ref_res = (s.to(torch.bfloat16).float() + res0[:T].float()).to(torch.bfloat16)
        xf = ref_res.float()
        ref_out = (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps) * w.float()).to(torch.bfloat16)
        row = {"T": T, "H": H, "world": world}
        for algo in (0, 1):
            fused = comms[algo]
            acc[:T].copy_(part)
            res[:T].copy_(res0[:T])
            fused.allreduce_norm(acc[:T], res[:T], w, eps, out[:T])
            torch.cuda.synchronize()
            assert ext().read_status() == 0, "bounded peer wait expired"
            assert float(acc[:T].abs().max()) == 0.0, "acc not cleared"
            d_res = float((res[:T].float() - ref_res.float()).abs().max())
            d_out = float((out[:T].float() - ref_out.float()).abs().max())
            # identical on every rank
            gathered = [torch.empty_like(out[:T]) for _ in range(world)]
            dist.all_gather(gathered, out[:T].contiguous())
            same = all(torch.equal(gathered[0], x) for x in gathered)
            row[f"algo{algo}_max_err_res"] = d_res
            row[f"algo{algo}_max_err_out"] = d_out
            row[f"algo{algo}_ranks_identical"] = same
            row[f"algo{algo}_us"] = timed(lambda: fused.allreduce_norm(acc[:T], res[:T], w, eps, out[:T]))

        def nccl():
            tp.all_reduce_(acc[:T])
            ops.add_rmsnorm(acc[:T], res[:T], w, eps, out=out[:T], clear_x=True)

        row["nccl_us"] = timed(nccl)
        b = T * H * 2
        row["roofline_us"] = 2 * (world - 1) / world * b / (LINK_GBS * 1e3)
        row["oneshot_bytes_us"] = (world - 1) * b / (LINK_GBS * 1e3)
        row["frac_roofline_algo0"] = row["roofline_us"] / row["algo0_us"]
        results.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
    assert ext().read_status() == 0
    for c in comms:
        c.close()
    dist.barrier()
    if rank == 0:
        print("done", flush=True)
    sys.stdout.flush()
    os._exit(0)


if __name__ == "__main__":
    main()
