"""Tensor parallelism on real GPUs: TP=2 must reproduce TP=1 logits and tokens.

Runs a small Llama (GPU-sized heads) from one HF checkpoint at TP=1 (in this process) and
TP=2 (two torchrun ranks) with NCCL collectives, the fused decode all-reduce, sequence
parallelism (NCCL and fused) and sampling data parallelism.  It compares

* the last-position logits of a prefill step of 6 x 40 tokens (the prefill path: SP when on)
  and of 6 x 16 tokens (96 rows: the decode-regime GEMMs and the fused all-reduce), relative
  error below 2e-2 and the same argmax, and
* the greedy tokens of a short generation whose decode batch shrinks as requests finish.

Skipped unless two CUDA devices are visible.
"""
import json
import os
import socket
import subprocess
import sys
import tempfile

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r'''
import json, os, sys, torch
sys.path.insert(0, sys.argv[1])
from vllm_neuron_b200.entrypoints import LLM
from vllm_neuron_b200.engine.sampling_params import SamplingParams
ckpt, out_path, fused, sp = sys.argv[2], sys.argv[3], sys.argv[4] == "1", sys.argv[5] == "1"
sdp = len(sys.argv) > 6 and sys.argv[6] == "1"
MAX_TOKENS = [12, 5, 9, 12, 3, 7]  # the decode batch shrinks as requests finish
torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
llm = LLM(ckpt, tensor_parallel_size=int(os.environ["WORLD_SIZE"]), max_num_seqs=8, max_model_len=256,
          num_gpu_blocks=256, max_num_batched_tokens=256, skip_tokenizer_init=True,
          additional_config={"b200_config": {"fused_comm": fused, "sequence_parallel": sp,
                                             "fused_sp": fused and sp, "sampling_dp": sdp}})
g = torch.Generator().manual_seed(0)
prompts = [torch.randint(0, 32000, (40,), generator=g).tolist() for _ in range(6)]
lg_long = llm.engine.prompt_logits(prompts)
lg_short = llm.engine.prompt_logits([p[:16] for p in prompts])
sps = [SamplingParams(temperature=0, max_tokens=n, ignore_eos=True) for n in MAX_TOKENS]
outs = llm.generate(prompts, sps)
from vllm_neuron_b200.ops._ext import ext
torch.cuda.synchronize()
assert ext().read_status() == 0, "a bounded peer wait expired"
assert llm.engine.model.sp_forwards > 0 or not sp, "sequence-parallel prefill did not run"
assert not sdp or llm.engine.runner.sampling_dp_steps > 0, "sampling DP did not run"
spf = llm.engine.model.sp_fused
assert not (fused and sp) or (spf is not None and spf.forwards > 0), "fused SP collectives did not run"
if int(os.environ["RANK"]) == 0:
    json.dump([o.outputs[0].token_ids for o in outs], open(out_path, "w"))
    torch.save({"long": lg_long, "short": lg_short}, out_path + ".pt")
llm.shutdown()
import torch.distributed as dist
dist.barrier(); dist.destroy_process_group()
'''


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def ckpt():
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=1024, num_hidden_layers=3, num_attention_heads=8, num_key_value_heads=4,
                      head_dim=128, intermediate_size=2048, vocab_size=32000, rms_norm_eps=1e-5,
                      rope_theta=500000.0, max_position_embeddings=1024, initializer_range=0.05)
    hf = LlamaForCausalLM(cfg).to(torch.bfloat16)
    d = tempfile.mkdtemp(prefix="tp_llama_")
    hf.save_pretrained(d, safe_serialization=True)
    return d


def _run_tp(ckpt, world, fused, sp=False, sdp=False):
    out = tempfile.mktemp(suffix=".json")
    script = tempfile.mktemp(suffix=".py")
    with open(script, "w") as f:
        f.write(WORKER)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", script, ROOT, ckpt, out, "1" if fused else "0", "1" if sp else "0", "1" if sdp else "0"]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return json.load(open(out)), torch.load(out + ".pt")


@pytest.mark.parametrize("fused,sp,sdp", [(False, False, False), (True, False, False), (False, True, False),
                                          (True, True, False), (True, False, True)])
def test_tp2_matches_tp1(ckpt, fused, sp, sdp):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 32000, (40,), generator=g).tolist() for _ in range(6)]
    sps = [SamplingParams(temperature=0, max_tokens=n, ignore_eos=True) for n in [12, 5, 9, 12, 3, 7]]
    llm = LLM(ckpt, max_num_seqs=8, max_model_len=256, num_gpu_blocks=256, max_num_batched_tokens=256,
              skip_tokenizer_init=True)
    ref_long = llm.engine.prompt_logits(prompts)
    ref_short = llm.engine.prompt_logits([p[:16] for p in prompts])
    ref = [o.outputs[0].token_ids for o in llm.generate(prompts, sps)]
    llm.shutdown()
    got, lg = _run_tp(ckpt, 2, fused, sp, sdp)
    for name, r in (("long", ref_long), ("short", ref_short)):
        t = lg[name]
        rel = float((t - r).norm() / r.norm())
        assert rel < 2e-2, (name, rel)
        # the same argmax, unless the reference's top two are a near tie (bf16 sums of the
        # partials in a different order may swap them)
        gap = r.max(-1).values - r.gather(-1, t.argmax(-1)[:, None]).squeeze(-1)
        assert bool((gap <= 1e-2 * r.abs().max()).all()), (name, gap)
    # The first generated token is the argmax of the "long" logits checked above (near ties
    # may swap); bf16 reduction order differs between TP sizes, so afterwards require most of
    # the generated tokens to match.
    same = sum(a == b for r, g2 in zip(ref, got) for a, b in zip(r, g2))
    assert same >= 0.8 * sum(len(r) for r in ref), (ref, got)


ADP_WORKER = r'''
import json, os, sys, torch
sys.path.insert(0, sys.argv[1])
from vllm_neuron_b200.entrypoints import LLM
from vllm_neuron_b200.engine.sampling_params import SamplingParams
ckpt, out_path = sys.argv[2], sys.argv[3]
torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
W = int(os.environ["WORLD_SIZE"])
llm = LLM(ckpt, tensor_parallel_size=1, max_num_seqs=8, max_model_len=256, num_gpu_blocks=256,
          max_num_batched_tokens=256, skip_tokenizer_init=True,
          additional_config={"neuron_config": {"mlp_dp_size": W, "embedding_dp_size": W, "lm_head_dp_size": W,
                                               "attention_dp_size": W}})
m = llm.engine.model
assert m.cdp_mlp and m.cdp_embed and m.cdp_lmh and m.cdp_attn and m.comp_tp.world == W and m.tp.world == 1
g = torch.Generator().manual_seed(0)
prompts = [torch.randint(0, 32000, (40,), generator=g).tolist() for _ in range(6)]
sps = [SamplingParams(temperature=0, max_tokens=n, ignore_eos=True) for n in [12, 5, 9, 12, 3, 7]]
outs = llm.generate(prompts, sps)
if int(os.environ["RANK"]) == 0:
    json.dump([o.outputs[0].token_ids for o in outs], open(out_path, "w"))
import torch.distributed as dist
dist.barrier(); dist.destroy_process_group()
'''


def test_component_dp2_matches_tp1(ckpt):
    """Component and attention DP over 2 GPUs: each GPU a data-parallel replica with the KV cache
    of its own requests; the MLP, the embedding, the LM head and the Q / O heads sharded over
    both GPUs (NCCL all-gathers of the replicas' rows, all-to-alls around attention,
    all-reduces)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 32000, (40,), generator=g).tolist() for _ in range(6)]
    sps = [SamplingParams(temperature=0, max_tokens=n, ignore_eos=True) for n in [12, 5, 9, 12, 3, 7]]
    llm = LLM(ckpt, max_num_seqs=8, max_model_len=256, num_gpu_blocks=256, max_num_batched_tokens=256,
              skip_tokenizer_init=True)
    ref = [o.outputs[0].token_ids for o in llm.generate(prompts, sps)]
    llm.shutdown()
    out = tempfile.mktemp(suffix=".json")
    script = tempfile.mktemp(suffix=".py")
    with open(script, "w") as f:
        f.write(ADP_WORKER)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", script, ROOT, ckpt, out]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = json.load(open(out))
    assert [len(x) for x in got] == [len(x) for x in ref]
    # the first token of every request is the argmax of its prefill logits; afterwards bf16 sums
    # in a different order (MLP partials over two GPUs, vocab-sliced LM head) may swap near ties
    # of this random model and a sequence then follows another path
    assert [x[0] for x in got] == [x[0] for x in ref], (ref, got)
    same = sum(a == b for r1, g2 in zip(ref, got) for a, b in zip(r1, g2))
    assert same >= 0.7 * sum(len(x) for x in ref), (ref, got)
