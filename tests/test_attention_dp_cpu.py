"""Attention data parallelism on CPU (gloo): the TP world splits into attention-DP replicas that
each run attention (heads over the replica's ranks, KV cache of their own requests) while the
MLP stays sharded over every rank; rows are gathered over the attention-DP group before each
MLP and each replica keeps its own after the all-reduce.  Greedy tokens equal TP=1."""
import multiprocessing as mp

import pytest

from tests._tiny import random_prompts, tiny_llama_checkpoint
from tests.test_tp_gloo_cpu import _free_port, _worker


@pytest.mark.parametrize("world,adp", [(2, 2), (4, 2)])
def test_attention_dp_matches_tp1(world, adp):
    ckpt, _ = tiny_llama_checkpoint()
    prompts = random_prompts(n=5, length=20, seed=21)  # odd count: replicas get 3 and 2
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=48).generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    extra = {"additional_config": {"neuron_config": {"attention_dp_size": adp}}}
    procs = [ctx.Process(target=_worker, args=(r, world, port, ckpt, prompts, q, world, extra))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        assert res[r][0] == ref, (r, res[r][0], ref)
