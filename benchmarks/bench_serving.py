"""Serving benchmark of the BASELINE model configurations through the public ``LLM`` API:
random-init weights of the named architecture, uniform-random token prompts, every request
generating exactly ``--output-len`` tokens (ignore_eos), all requests submitted at once
(continuous batching, chunked prefill).  Reports output tok/s (device-timed with CUDA events
around the whole run, max over ranks), p50 TTFT and p50 TPOT (host clocks).

    python benchmarks/bench_serving.py --model gpt-oss-20b [--num-prompts 32 --input-len 2048 --output-len 512]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_serving.py --model ... --tp N

Models (shapes of the BASELINE configurations):
  llama3-8b     32 layers, hidden 4096, 32/8 heads x 128, FFN 14336, vocab 128256
  gpt-oss-20b   24 layers, hidden 2880, 64/8 heads x 64, sliding 128 / full alternating, sinks,
                32 experts top-4 (FFN 2880), vocab 201088
  qwen3.6-a3b   40 layers (3 gated-DeltaNet : 1 gated attention), hidden 2048, attention 16/2 x
                256, DeltaNet 16 key / 32 value heads x 128, conv 4, 256 experts top-8 (FFN 512)
                + 1 shared expert, vocab 248320
  llama3-70b    80 layers, hidden 8192, 64/8 heads x 128, FFN 28672, vocab 128256
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

MODELS = {
    "llama3-8b": dict(
        cfg={"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
             "num_hidden_layers": 32, "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128,
             "intermediate_size": 14336, "vocab_size": 128256, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
             "max_position_embeddings": 8192},
        workload=(64, 1024, 256)),
    "gpt-oss-20b": dict(
        cfg={"architectures": ["GptOssForCausalLM"], "model_type": "gpt_oss", "hidden_size": 2880,
             "num_hidden_layers": 24, "num_attention_heads": 64, "num_key_value_heads": 8, "head_dim": 64,
             "intermediate_size": 2880, "num_local_experts": 32, "num_experts_per_tok": 4,
             "vocab_size": 201088, "rms_norm_eps": 1e-5, "sliding_window": 128,
             "layer_types": ["sliding_attention", "full_attention"] * 12, "swiglu_limit": 7.0,
             "max_position_embeddings": 131072, "rope_theta": 150000.0,
             "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                              "truncate": False, "original_max_position_embeddings": 4096}},
        workload=(32, 2048, 512)),
    "qwen3.6-a3b": dict(
        cfg={"architectures": ["Qwen3_5MoeForCausalLM"], "model_type": "qwen3_5_moe_text", "hidden_size": 2048,
             "num_hidden_layers": 40, "num_attention_heads": 16, "num_key_value_heads": 2, "head_dim": 256,
             "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
             "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4, "num_experts": 256,
             "num_experts_per_tok": 8, "moe_intermediate_size": 512, "shared_expert_intermediate_size": 512,
             "norm_topk_prob": True, "vocab_size": 248320, "rms_norm_eps": 1e-6,
             "layer_types": (["linear_attention"] * 3 + ["full_attention"]) * 10,
             "rope_parameters": {"rope_type": "default", "rope_theta": 10000000.0, "partial_rotary_factor": 0.25},
             "max_position_embeddings": 32768},
        workload=(64, 4096, 256), quant="fp8_block"),
    "llama3-70b": dict(
        cfg={"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 8192,
             "num_hidden_layers": 80, "num_attention_heads": 64, "num_key_value_heads": 8, "head_dim": 128,
             "intermediate_size": 28672, "vocab_size": 128256, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
             "max_position_embeddings": 16384},
        workload=(16, 8192, 512), quant="fp8_block", mnbt=4096, sp=True),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gpt-oss-20b", choices=sorted(MODELS))
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--num-prompts", type=int, default=None)
    ap.add_argument("--input-len", type=int, default=None)
    ap.add_argument("--output-len", type=int, default=None)
    ap.add_argument("--max-num-batched-tokens", type=int, default=None)
    ap.add_argument("--warmup-prompts", type=int, default=4)
    ap.add_argument("--json", default=None)
    ap.add_argument("--quant", default="auto", choices=["auto", "none", "fp8_static", "fp8_block", "mxfp8"],
                    help="fp8_static: W8A8 FP8 projections (random weights quantized per tensor); "
                         "fp8_block: 128 x 128 block-scaled FP8 weights, bf16 activations; mxfp8: "
                         "MXFP8 projections (e8m0 scale per 32, block-scaled tensor cores); auto: the "
                         "configuration's own (fp8_block for llama3-70b and qwen3.6-a3b)")
    ap.add_argument("--sp", action="store_true", help="sequence-parallel prefill (TP > 1)")
    ap.add_argument("--fp8-block-act", choices=["fp8", "bf16"], default=None,
                    help="block-FP8 decode projections: W8A8 (fp8 activations) or W8A16")
    ap.add_argument("--baseline", action="store_true",
                    help="NCCL + cuBLAS build of the same engine (no fused kernels, library GEMMs)")
    a = ap.parse_args()

    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    rank, world = ps.init_distributed(timeout_s=600)
    if world > 1:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    m = MODELS[a.model]
    P, IN, OUT = m["workload"]
    P = a.num_prompts or P
    IN = a.input_len or IN
    OUT = a.output_len or OUT
    max_len = IN + OUT + 16
    blocks = P * ((max_len + 15) // 16) + 64
    nc = {}
    quant = m.get("quant") if a.quant == "auto" else (None if a.quant == "none" else a.quant)
    if quant:
        nc["quantization"] = quant
    if a.sp or (m.get("sp") and world > 1):
        nc["sequence_parallel"] = True
    if a.baseline:
        nc.update(fused_comm=False, use_cublas_baseline=True)
    if a.fp8_block_act:
        nc["fp8_block_activations"] = a.fp8_block_act
    mnbt = a.max_num_batched_tokens or m.get("mnbt", 8192)
    llm = LLM(dict(m["cfg"]), tensor_parallel_size=world, max_num_seqs=P, max_model_len=max_len,
              max_num_batched_tokens=mnbt, load_format="dummy", num_gpu_blocks=blocks,
              skip_tokenizer_init=True, seed=0, additional_config={"neuron_config": nc} if nc else None)
    vocab = m["cfg"]["vocab_size"]
    g = torch.Generator().manual_seed(7)
    prompts = torch.randint(0, vocab, (P, IN), generator=g).tolist()
    # warm-up (kernels, graphs, allocator)
    llm.generate(prompts[:a.warmup_prompts], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    sp = SamplingParams(temperature=0.0, max_tokens=OUT, ignore_eos=True)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    outs = llm.generate(prompts, sp)
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ttft = [o.metrics["first_token_time"] - o.metrics["arrival_time"] for o in outs]
    tpot = [(o.metrics["finish_time"] - o.metrics["first_token_time"]) / max(1, len(o.outputs[0].token_ids) - 1)
            for o in outs]
    assert all(len(o.outputs[0].token_ids) == OUT for o in outs)
    res = {"model": a.model, "tp": world, "num_prompts": P, "input_len": IN, "output_len": OUT,
           "output_tok_s": P * OUT / (ms / 1e3), "wall_s": wall, "device_s": ms / 1e3,
           "p50_ttft_ms": float(np.median(ttft)) * 1e3, "p50_tpot_ms": float(np.median(tpot)) * 1e3,
           "dtype": "bf16" + ({"fp8_static": " activations, fp8 W8A8 projections",
                               "fp8_block": (" activations, 128x128 block-scaled fp8 weights (decode: "
                                             + ("W8A16" if a.fp8_block_act == "bf16" else
                                                "W8A8, 1x128 fp8 activation blocks") + ")"),
                               "mxfp8": " activations, MXFP8 W8A8 projections (e4m3, e8m0 per 32)"}.get(quant, "")),
           "sp": bool(nc.get("sequence_parallel")), "max_num_batched_tokens": mnbt,
           "build": "nccl+cublas baseline" if a.baseline else "fused sm_100a",
           "data": "synthetic prompts, random-init weights"}
    if rank == 0:
        print(json.dumps(res), flush=True)
        if a.json:
            with open(a.json, "w") as f:
                json.dump(res, f)
    sys.stdout.flush()
    os._exit(0)


if __name__ == "__main__":
    main()
