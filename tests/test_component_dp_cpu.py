"""Component and attention data parallelism on CPU (gloo): data-parallel replicas that step in
lockstep while the chosen components (dense MLP, embedding, LM head, the Q / O heads of
attention) shard their weights over every rank of every replica; per component the replicas'
rows are gathered over the DP column (all-to-all for attention), each rank computes its shard
and the replicas keep their own rows.  The KV cache of each replica's requests stays on the
replica.  Greedy tokens equal TP=1."""
import multiprocessing as mp

import pytest

from tests._tiny import random_prompts, tiny_llama_checkpoint
from tests.test_tp_gloo_cpu import _free_port, _worker

ALL = {"mlp_dp_size": 2, "embedding_dp_size": 2, "lm_head_dp_size": 2}


@pytest.mark.parametrize("world,tp,opts", [(2, 1, {"mlp_dp_size": 2}), (2, 1, ALL), (4, 2, ALL),
                                           (4, 2, {"lm_head_dp_size": 2}),
                                           (2, 1, {"attention_dp_size": 2}),
                                           (4, 2, dict(ALL, attention_dp_size=2)),
                                           # four replicas, components shared by pairs or by all
                                           (4, 1, {"mlp_dp_size": 2, "attention_dp_size": 4,
                                                   "lm_head_dp_size": 2, "embedding_dp_size": 4})])
def test_component_dp_matches_tp1(world, tp, opts):
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
    extra = {"additional_config": {"neuron_config": dict(opts)}}
    procs = [ctx.Process(target=_worker, args=(r, world, port, ckpt, prompts, q, tp, extra))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        assert res[r][0] == ref, (r, res[r][0], ref)


def test_component_dp_refusals():
    from vllm_neuron_b200.config import B200Config

    with pytest.raises(ValueError):
        from vllm_neuron_b200.entrypoints import LLM

        ckpt, _ = tiny_llama_checkpoint()
        LLM(ckpt, device="cpu", max_num_seqs=4, max_model_len=64, num_gpu_blocks=16,
            additional_config={"neuron_config": {"mlp_dp_size": 2}})  # one process: no replicas
    assert B200Config.from_dict({"mlp_dp_size": 2}).mlp_dp_size == 2


def test_attention_dp_on_moe_model():
    """Attention / embedding / LM-head DP on a Qwen3-MoE decoder (experts stay per replica)
    equal the single-process tokens; mlp_dp_size is refused for expert MLPs."""
    from tests.test_ep_a2a_cpu import _qwen_moe_ckpt

    ckpt = _qwen_moe_ckpt()
    prompts = random_prompts(n=3, length=12, vocab=512, seed=5)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=48).generate(prompts, SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    extra = {"additional_config": {"neuron_config": {"attention_dp_size": 2, "embedding_dp_size": 2,
                                                     "lm_head_dp_size": 2}}}
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ckpt, prompts, q, 1, extra)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        # the worker generates 8 tokens; compare the first 6
        assert [t[:6] for t in res[r][0]] == ref, (r, res[r][0], ref)


def test_attention_dp_on_gpt_oss():
    """GPT-OSS (qkv and o biases, sinks, sliding windows) with attention / embedding / LM-head
    DP over two replicas equals the single-process tokens."""
    from tests.test_gpt_oss_cpu import _tiny_gpt_oss

    ckpt, _ = _tiny_gpt_oss()
    prompts = random_prompts(n=3, length=14, vocab=512, seed=6)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=48).generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    extra = {"additional_config": {"neuron_config": {"attention_dp_size": 2, "embedding_dp_size": 2,
                                                     "lm_head_dp_size": 2}}}
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ckpt, prompts, q, 1, extra)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        assert res[r][0] == ref, (r, res[r][0], ref)


def test_vocab_dp_on_hybrid_and_refusal():
    """Embedding / LM-head DP on the Qwen3.5/3.6-style hybrid (DeltaNet and gated attention stay
    per replica) equals the single-process tokens; attention DP is refused for it."""
    from tests.test_hybrid_cpu import _tiny_hybrid

    d, _ = _tiny_hybrid()
    prompts = random_prompts(n=3, length=12, vocab=512, seed=8)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    kw = dict(device="cpu", dtype="float32", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=48)
    ref = LLM(d, **kw).generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    for opts, ok in (({"embedding_dp_size": 2, "lm_head_dp_size": 2}, True), ({"attention_dp_size": 2}, False)):
        q = ctx.Queue()
        port = _free_port()
        extra = {"dtype": "float32", "additional_config": {"neuron_config": opts}}
        procs = [ctx.Process(target=_worker, args=(r, 2, port, d, prompts, q, 1, extra)) for r in range(2)]
        for p in procs:
            p.start()
        res = dict(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=60)
        for r in range(2):
            if ok:
                assert not isinstance(res[r], str), res[r]
                assert res[r][0] == ref, (r, res[r][0], ref)
            else:
                assert isinstance(res[r], str) and "not supported" in res[r], res[r]
