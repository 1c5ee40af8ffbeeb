"""Device time of one serving step of Llama-3-8B (random weights) on one GPU, without host
overhead: a decode step of B sequences at context L replayed from its CUDA graph, and one
eager prefill chunk of T tokens.  Also reports the host time of batch preparation.

    python benchmarks/bench_step.py [--batch 64] [--ctx 1152] [--chunk 8192] [--layers 32]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_step.py ...   (TP=N)
    python benchmarks/bench_step.py --emulate-tp N     (one GPU runs rank 0's share of TP=N)

With TP, times are the maximum over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from benchmarks.bench_serving import MODELS  # noqa: E402
from vllm_neuron_b200.engine.request import Request  # noqa: E402
from vllm_neuron_b200.engine.sampling_params import SamplingParams  # noqa: E402
from vllm_neuron_b200.engine.scheduler import ScheduledRequest, SchedulerOutput  # noqa: E402
from vllm_neuron_b200.entrypoints import LLM  # noqa: E402


def decode_timeline(replay, n: int) -> list[dict]:
    """Per-kernel share of ``n`` replays of a decode graph: kernels sorted by start; each one's
    increment is how far its end moves the running maximum end time (launches that overlap under
    programmatic dependent launch are charged only for what they add to the step)."""
    import re
    from collections import OrderedDict

    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            replay()
        torch.cuda.synchronize()
    ev = sorted((e.time_range.start, e.time_range.end, e.name) for e in prof.events()
                if e.device_type == torch.autograd.DeviceType.CUDA)
    if not ev:
        return []
    agg: OrderedDict[str, list] = OrderedDict()
    last = ev[0][0]
    for s0, e1, name in ev:
        inc = max(0.0, e1 - last)
        last = max(last, e1)
        key = re.sub(r"\(.*", "", name)[:80]
        a = agg.setdefault(key, [0, 0.0])
        a[0] += 1
        a[1] += inc
    total = sum(v[1] for v in agg.values()) or 1.0
    return [{"kernel": k, "launches_per_step": c / n, "us_per_step": t / n, "share": t / total}
            for k, (c, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b", choices=sorted(MODELS))
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1152)
    ap.add_argument("--chunk", type=int, default=8192)
    ap.add_argument("--layers", type=int, default=None, help="default: the model's layer count")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", type=str, default=None)
    ap.add_argument("--no-fused", action="store_true", help="TP: NCCL all-reduce instead of the fused kernel")
    ap.add_argument("--sp", action="store_true", help="TP prefill: sequence parallelism (fused unless --no-fused)")
    ap.add_argument("--emulate-tp", type=int, default=1,
                    help="one GPU runs rank 0's share of TP=N with local no-op collectives (profiling only)")
    ap.add_argument("--timeline", action="store_true",
                    help="break the decode step's graph replay into per-kernel increments (torch "
                         "profiler trace of 10 replays; a kernel's increment is how far it moves the "
                         "last kernel end, so PDL overlap is not double-counted)")
    ap.add_argument("--profile-once", action="store_true",
                    help="run one decode replay and one prefill chunk inside NVTX ranges "
                         "'decode_step' / 'prefill_chunk' (for an ncu launch list)")
    a = ap.parse_args()
    from vllm_neuron_b200.parallel import state as ps

    rank, world = ps.init_distributed(timeout_s=300)
    if world > 1:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    a.layers = min(a.layers or MODELS[a.model]["cfg"]["num_hidden_layers"], MODELS[a.model]["cfg"]["num_hidden_layers"])
    cfg = dict(MODELS[a.model]["cfg"], num_hidden_layers=a.layers)
    if "layer_types" in cfg:
        cfg["layer_types"] = cfg["layer_types"][:a.layers]
    B, L = a.batch, a.ctx
    max_len = max(L + 64, 2048)
    blocks = B * (max_len // 16 + 1) + 64
    if a.emulate_tp > 1:
        from vllm_neuron_b200.engine.llm_engine import EngineArgs, LLMEngine
        from vllm_neuron_b200.parallel.comm import EmulatedRankComm

        eng = LLMEngine(EngineArgs(model=cfg, max_num_seqs=B, max_model_len=max_len,
                                   max_num_batched_tokens=a.chunk, load_format="dummy",
                                   num_gpu_blocks=blocks), tp=EmulatedRankComm(a.emulate_tp))
    else:
        llm = LLM(cfg, tensor_parallel_size=world,
                  additional_config={"b200_config": {"fused_comm": not a.no_fused,
                                                     "sequence_parallel": a.sp}},
                  max_num_seqs=B, max_model_len=max_len, max_num_batched_tokens=a.chunk,
                  load_format="dummy", num_gpu_blocks=blocks, skip_tokenizer_init=True)
        eng = llm.engine
    runner = eng.runner
    sp = SamplingParams(temperature=0.0, max_tokens=1 << 20, ignore_eos=True)
    # Fake B running requests at context L with contiguous block ids.
    reqs = []
    nb = (L + 1 + 15) // 16
    for i in range(B):
        r = Request(str(i), list(np.random.randint(0, 1000, L)), sp)
        r.output_token_ids = [1]
        r.num_computed_tokens = L
        r.slot = i
        r.block_ids = list(range(1 + i * nb, 1 + (i + 1) * nb))
        reqs.append(r)
    out = SchedulerOutput([ScheduledRequest(r, L, 1, True) for r in reqs], B)
    res = {}
    if a.profile_once:
        bucket = min(b for b in runner.graphs if b >= B)
        g = runner.graphs[bucket][0]
        lay_b, buf_b = runner.graphs[bucket][1], runner.graphs[bucket][2]
        runner._pack(out, lay_b, pad_B=bucket)
        buf_b.copy_(runner.host_buf[:lay_b.total])
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_step")
        g.replay()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        T = a.chunk
        n_seq = max(1, T // 1024)
        per = T // n_seq
        nb2 = (per + 15) // 16
        preqs = []
        for i in range(n_seq):
            r = Request("p%d" % i, list(np.random.randint(0, 1000, per)), sp)
            r.slot = B + i
            r.block_ids = list(range(1 + i * nb2, 1 + (i + 1) * nb2))
            preqs.append(r)
        pout = SchedulerOutput([ScheduledRequest(r, 0, per, True) for r in preqs], per * n_seq)
        torch.cuda.nvtx.range_push("prefill_chunk")
        runner.execute(pout)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        print("profile-once done", flush=True)
        return
    # host preparation cost
    t0 = time.perf_counter()
    for _ in range(50):
        runner.execute(out)
    torch.cuda.synchronize()
    res["decode_step_with_host_ms"] = (time.perf_counter() - t0) / 50 * 1e3
    g, lay, buf, tok, lp, splits = runner.graphs[min(b for b in runner.graphs if b >= B)]
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    res["decode_step_gpu_ms"] = e0.elapsed_time(e1) / a.iters
    res["attn_splits"] = splits
    if a.timeline:
        res["decode_timeline"] = decode_timeline(g.replay, 10)
    t0 = time.perf_counter()
    for _ in range(200):
        runner._pack(out, lay, pad_B=min(b for b in runner.graphs if b >= B))
    res["pack_host_ms"] = (time.perf_counter() - t0) / 200 * 1e3
    # prefill chunk
    T = a.chunk
    n_seq = max(1, T // 1024)
    per = T // n_seq
    preqs = []
    nb2 = (per + 15) // 16
    for i in range(n_seq):
        r = Request("p%d" % i, list(np.random.randint(0, 1000, per)), sp)
        r.slot = B + i
        r.block_ids = list(range(1 + i * nb2, 1 + (i + 1) * nb2))
        preqs.append(r)
    pout = SchedulerOutput([ScheduledRequest(r, 0, per, True) for r in preqs], per * n_seq)
    runner.execute(pout)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(3):
        runner.execute(pout)
    e1.record()
    torch.cuda.synchronize()
    res["prefill_chunk_ms"] = e0.elapsed_time(e1) / 3
    res["prefill_tokens"] = per * n_seq
    flops = 2 * 7.5e9 * per * n_seq * a.layers / 32  # Llama-3-8B dense FLOPs (other models: ignore)
    res["prefill_tflops_dense_only"] = flops / (res["prefill_chunk_ms"] * 1e9)
    res.update(batch=B, ctx=L, layers=a.layers, tp=world, emulated_tp=a.emulate_tp)
    if world > 1:
        import torch.distributed as dist

        keys = [k for k, v in res.items() if k.endswith("_ms")]
        t = torch.tensor([res[k] for k in keys], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        for k, v in zip(keys, t.tolist()):
            res[k] = v
        res["prefill_tflops_dense_only"] = flops / (res["prefill_chunk_ms"] * 1e9)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if a.json and rank == 0:
        with open(a.json, "w") as f:
            json.dump(res, f)
    sys.stdout.flush()
    # Skip interpreter teardown (IPC mappings and NCCL communicators are released by the
    # process exit); every rank has finished its collectives above.
    os._exit(0)


if __name__ == "__main__":
    main()
