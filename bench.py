"""Headline benchmark: output tok/s of Llama-3-8B serving, 64 concurrent requests of 1024
random input tokens generating 256 tokens each (ignore_eos), tensor parallel over the GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|baseline|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

With N > 1 prefill runs sequence-parallel (fused reduce-scatter / all-gather GEMMs) and decode
uses the fused all-reduce + RMSNorm kernel.  After the fused build, the same process builds
the NCCL + cuBLAS version of the same engine (dense projections on cuBLAS through torch.mm,
collectives on NCCL) and times it on the same workload: ``baseline_value`` / ``baseline_e2e``
(``--baseline-steps`` waves; ``--no-baseline`` skips it).

One *step* is one full wave of the workload: all 64 requests are submitted at once and
served to completion with continuous batching and chunked prefill (8192-token budget).
``value`` is device-timed: CUDA events around exactly K waves, bracketed by a barrier and a
synchronize on both sides, maximum over ranks.  ``e2e`` repeats the measurement through the
public API (``LLM.generate`` with token-id prompts taken from pinned host memory; every
engine step copies its inputs host->device and reads the sampled tokens device->host).
Weights are random-init (N(0, 0.02)) with the exact Llama-3-8B shapes; inputs are uniform
random token ids.  16 GB of weights are streamed every step, far more than L2 (126 MB).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "output tok/s per box (Llama-3-8B TP8, 1k in/256 out, conc 64); p50 TTFT, p50 TPOT"
# The reference's published Llama-3.1-8B TP8 output throughput on trn2.48xlarge (512 in / 128
# out, concurrency 2): a different workload, kept only as the order-of-magnitude context the
# driver divides by.
PUBLISHED_TOK_S = 184.44

LLAMA3_8B = {
    "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
    "num_hidden_layers": 32, "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128,
    "intermediate_size": 14336, "vocab_size": 128256, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
    "max_position_embeddings": 8192, "tie_word_embeddings": False, "eos_token_id": 128001,
}


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args):
    """The reference (vllm-neuron) runs only on AWS Trainium through libtorch_neuronx_lite."""
    why = None
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "vllm_neuron")):
        why = "reference not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref_dir)
        try:
            import importlib.util

            import vllm_neuron  # noqa: F401
            missing = [m for m in ("libtorch_neuronx_lite", "nkilib", "neuronxcc")
                       if importlib.util.find_spec(m) is None]
            why = ("vllm-neuron is installed (baseline/_ref) but executes only on AWS Neuron "
                   "devices through libtorch_neuronx_lite/nkilib/neuronx-cc; missing here: "
                   + (", ".join(missing) if missing else "a Neuron device"))
        except Exception as e:
            why = f"vllm-neuron import failed: {type(e).__name__}: {str(e)[:160]}"
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)


def measure(llm, waves, args, steps: int, warmup: int, e2e_steps: int | None, world: int, dev) -> dict:
    """Serve ``warmup`` untimed waves, then time exactly ``steps`` waves (CUDA events, barrier +
    synchronize on both sides, max over ranks), then ``e2e_steps`` waves through ``LLM.generate``."""
    import torch
    import torch.distributed as dist

    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.ops._ext import ext

    eng = llm.engine
    P, OUT = args.num_prompts, args.output_len
    sp = SamplingParams(temperature=0.0, max_tokens=OUT, ignore_eos=True)
    local = dev.index

    def run_wave(i: int):
        prompts = waves[i % 2].tolist()
        t0 = time.perf_counter()
        for j, p in enumerate(prompts):
            eng.add_request(p, sp, request_id=f"w{i}-{j}", arrival_time=t0)
        return eng.run_until_done()

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(warmup):
        run_wave(i)
    torch.cuda.synchronize()
    barrier()

    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                          if os.environ.get("CUDA_VISIBLE_DEVICES") else local)
    clocks.start()
    r0 = eng.runner
    launches0 = ext().launch_count()
    replayed0 = r0.replayed_kernels
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    ev0.record()
    ttft, tpot = [], []
    for i in range(steps):
        for r in run_wave(warmup + i):
            ttft.append(r.first_token_time - r.arrival_time)
            if len(r.output_token_ids) > 1:
                tpot.append((r.finish_time - r.first_token_time) / (len(r.output_token_ids) - 1))
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    gpu_launches = (ext().launch_count() - launches0) + (r0.replayed_kernels - replayed0)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = steps * P * OUT / (ms / 1e3)

    # ---- end to end through the public API
    e2e = None
    if e2e_steps:
        h2d0, d2h0 = r0.h2d_bytes, r0.d2h_bytes
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            outs = llm.generate(waves[i % 2], sp)
            assert len(outs) == P and all(len(o.outputs[0].token_ids) == OUT for o in outs)
        torch.cuda.synchronize()
        barrier()
        dt = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([dt], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        e2e = {"value": e2e_steps * P * OUT / dt, "unit": "tok/s",
               "h2d_bytes_per_step": int((r0.h2d_bytes - h2d0) / e2e_steps),
               "d2h_bytes_per_step": int((r0.d2h_bytes - d2h0) / e2e_steps),
               "api": "vllm_neuron_b200.entrypoints.LLM.generate"}
    return {"value": value, "ms": ms, "steps": steps, "warmup": warmup, "clocks": clk, "e2e": e2e,
            "gpu_launches": int(gpu_launches),
            "p50_ttft_ms": round(float(np.median(ttft)) * 1e3, 2) if ttft else None,
            "p50_tpot_ms": round(float(np.median(tpot)) * 1e3, 3) if tpot else None,
            "graph_replays": r0.num_graph_replays, "eager_steps": r0.num_eager_steps,
            "device_status": int(ext().read_status())}


def build_llm(cfg, args, world: int, sp_on: bool, baseline: bool):
    from vllm_neuron_b200.entrypoints import LLM

    P, IN, OUT = args.num_prompts, args.input_len, args.output_len
    max_len = IN + OUT + 16
    blocks = P * ((max_len + 15) // 16) + 64
    opts = {"sequence_parallel": sp_on}
    if sp_on and not baseline and args.fused_sp:
        opts["fused_sp"] = True
    if baseline:  # NCCL collectives + cuBLAS projections, same engine, kernels and schedule otherwise
        opts.update(fused_comm=False, use_cublas_baseline=True)
    return LLM(cfg, tensor_parallel_size=world, max_num_seqs=P, max_model_len=max_len,
               max_num_batched_tokens=args.max_num_batched_tokens, block_size=16, load_format="dummy",
               num_gpu_blocks=blocks, seed=0, skip_tokenizer_init=True,
               additional_config={"b200_config": opts})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "baseline", "reference"],
                    help="b200: fused sm_100a build (and, unless --no-baseline, the NCCL + cuBLAS "
                         "build of the same engine after it); baseline: only the NCCL + cuBLAS build")
    ap.add_argument("--num-prompts", type=int, default=64)
    ap.add_argument("--input-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--max-num-batched-tokens", type=int, default=8192)
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-baseline", action="store_true")
    ap.add_argument("--baseline-steps", type=int, default=5,
                    help="timed waves of the NCCL + cuBLAS build (at most --steps)")
    ap.add_argument("--layers", type=int, default=None, help="debug only: fewer layers (invalid for reporting)")
    ap.add_argument("--fused-sp", action="store_true",
                    help="sequence-parallel prefill on the fused GEMM -> reduce-scatter / all-gather -> GEMM "
                         "kernels over NVLink peer memory (default: NCCL collectives)")
    ap.add_argument("--sp", choices=["auto", "on", "off"], default="auto",
                    help="sequence-parallel prefill (auto: on when N > 1)")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)

    import gc

    import torch

    from vllm_neuron_b200.parallel import state as ps

    rank, world = ps.init_distributed(timeout_s=600)
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = dict(LLAMA3_8B)
    if args.layers:
        cfg["num_hidden_layers"] = args.layers
    P, IN, OUT = args.num_prompts, args.input_len, args.output_len
    g = torch.Generator().manual_seed(1234)
    # Token-id prompts live in pinned host memory (one tensor per wave).
    waves = [torch.randint(0, cfg["vocab_size"], (P, IN), generator=g, dtype=torch.int32).pin_memory()
             for _ in range(2)]
    sp_on = args.sp == "on" or (args.sp == "auto" and world > 1)
    e2e_steps = None if args.no_e2e else (args.e2e_steps or args.steps)

    main_baseline = args.impl == "baseline"
    llm = build_llm(cfg, args, world, sp_on, baseline=main_baseline)
    eng = llm.engine
    res = measure(llm, waves, args, args.steps, args.warmup, e2e_steps, world, dev)
    fused_tp = eng.model.tp_fused is not None
    sp_info = {"on": sp_on, "fused": eng.model.sp_fused is not None, "prefill_forwards": eng.model.sp_forwards}
    base = None
    if args.impl == "b200" and not args.no_baseline:
        llm.shutdown()
        del llm, eng
        gc.collect()
        torch.cuda.empty_cache()
        bl = build_llm(cfg, args, world, sp_on, baseline=True)
        ks = max(1, min(args.steps, args.baseline_steps))
        b = measure(bl, waves, args, ks, min(args.warmup, 3), None if args.no_e2e else ks, world, dev)
        base = {"value": round(b["value"], 2), "e2e": b["e2e"]["value"] if b["e2e"] else None,
                "ms_per_step": round(b["ms"] / ks, 3), "steps": ks, "warmup": b["warmup"],
                "p50_ttft_ms": b["p50_ttft_ms"], "p50_tpot_ms": b["p50_tpot_ms"], "clocks": b["clocks"],
                "build": "same engine; dense projections on cuBLAS (torch.mm), collectives on NCCL "
                         "(all-reduce / reduce-scatter + all-gather), no fused kernels",
                "device_status": b["device_status"]}
        llm = bl

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(res["value"], 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(res["ms"] / args.steps, 3),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": round(res["value"] / PUBLISHED_TOK_S, 3), "dtype": "bf16",
            "data": "synthetic (uniform random token ids; random-init N(0,0.02) Llama-3-8B weights)",
            "config": {"model": "Llama-3-8B architecture" + (f" ({args.layers} layers: DEBUG)" if args.layers else ""),
                       "global_batch": P, "seq_len": IN + OUT, "input_len": IN, "output_len": OUT,
                       "concurrency": P, "parallelism": f"tp{world}" + ("+sp" if sp_on else ""), "block_size": 16,
                       "max_num_batched_tokens": args.max_num_batched_tokens,
                       "l2": "inputs larger than L2 (16 GB of weights + KV streamed per step)"},
            "p50_ttft_ms": res["p50_ttft_ms"], "p50_tpot_ms": res["p50_tpot_ms"],
            "clocks": res["clocks"], "e2e": res["e2e"], "gpu_launches": res["gpu_launches"],
            "graph_replays": res["graph_replays"], "eager_steps": res["eager_steps"],
            "device_status": res["device_status"],
            "fused_tp_comm": fused_tp, "sequence_parallel": sp_info,
        }
        if main_baseline:
            line["impl"] = "baseline"
        if base is not None:
            line["baseline_value"] = base["value"]
            line["baseline_e2e"] = base["e2e"]
            line["baseline"] = base
        print(json.dumps(line), flush=True)
    if world > 1:
        # Every rank has finished its collectives; leave without tearing down the process group
        # (graph-held communicators otherwise make the exit wait).
        import torch.distributed as dist

        dist.barrier()
        sys.stdout.flush()
        os._exit(0)
    llm.shutdown()


if __name__ == "__main__":
    main()
