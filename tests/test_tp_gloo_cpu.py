"""Tensor parallelism on CPU: two gloo ranks serve the tiny Llama with TP=2 (sharded qkv /
o / gate_up / down, vocab-sharded embedding and LM head, all-reduce + all-gather) and must
produce the same greedy tokens as TP=1."""
import multiprocessing as mp
import os
import socket

from tests._tiny import random_prompts, tiny_llama_checkpoint


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, ckpt, prompts, q, tp=None, extra=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch

    torch.set_num_threads(1)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    try:
        llm = LLM(ckpt, tensor_parallel_size=tp or world, device="cpu", max_num_seqs=8, max_model_len=128,
                  num_gpu_blocks=64, **dict(dict(max_num_batched_tokens=48), **(extra or {})))
        outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
        toks = [o.outputs[0].token_ids for o in outs]
        q.put((rank, (toks, llm.engine.model.sp_forwards) if extra else toks))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        ps.destroy_parallel_state()


def test_tp2_matches_tp1():
    ckpt, _ = tiny_llama_checkpoint()
    prompts = random_prompts(n=3, length=20, seed=11)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=48).generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ckpt, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == ref, res[0]
    assert res[1] == ref, res[1]


def test_tp2_sequence_parallel_matches_tp1():
    """Prefill with the residual stream sharded over tokens (reduce-scatter / all-gather, odd
    token counts padded to the TP size) gives the TP=1 tokens."""
    ckpt, _ = tiny_llama_checkpoint()
    prompts = random_prompts(n=3, length=71, seed=5)  # one 213-token prefill step (> decode path)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=256).generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    extra = {"additional_config": {"neuron_config": {"sequence_parallel": True}}, "max_num_batched_tokens": 256}
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ckpt, prompts, q, None, extra)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        toks, n_sp = res[r]
        assert toks == ref, toks
        assert n_sp >= 1


def test_dp2_matches_single_replica():
    """Two data-parallel replicas (TP=1 each) split the requests and gather the outputs."""
    ckpt, _ = tiny_llama_checkpoint()
    prompts = random_prompts(n=5, length=16, seed=12)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=48).generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ckpt, prompts, q, 1)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == ref, res[0]
    assert res[1] == ref, res[1]


def _sdp_worker(rank, world, port, ckpt, prompts, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch

    torch.set_num_threads(1)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    try:
        llm = LLM(ckpt, tensor_parallel_size=world, device="cpu", max_num_seqs=8, max_model_len=128,
                  num_gpu_blocks=64, max_num_batched_tokens=48,
                  additional_config={"neuron_config": {"sampling_dp": True}})
        sps = [SamplingParams(temperature=0.8 if i % 2 else 0.0, top_k=50, seed=100 + i, max_tokens=6,
                              ignore_eos=True) for i in range(len(prompts))]
        outs = llm.generate(prompts, sps)
        q.put((rank, ([o.outputs[0].token_ids for o in outs], llm.engine.runner.sampling_dp_steps)))
    except Exception:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        ps.destroy_parallel_state()


def test_sampling_dp_matches_replicated_sampling():
    """TP=2 with sampling data parallelism (each rank samples half the rows after an all-to-all
    of the vocab-sharded logits): greedy and seeded random rows equal the TP=1 engine's."""
    ckpt, _ = tiny_llama_checkpoint()
    prompts = random_prompts(n=5, length=12, seed=21)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    sps = [SamplingParams(temperature=0.8 if i % 2 else 0.0, top_k=50, seed=100 + i, max_tokens=6,
                          ignore_eos=True) for i in range(len(prompts))]
    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=48).generate(prompts, sps)
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sdp_worker, args=(r, 2, port, ckpt, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
        toks, steps = res[r]
        assert steps > 0 and toks == ref, (r, toks, ref)
