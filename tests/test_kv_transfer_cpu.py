"""Disaggregated prefill / decode on CPU: rank 0 is a prefill engine (kv_producer) that samples
the first tokens of each request and hands the request with its KV cache to rank 1, a decode
engine (kv_consumer) that finishes it.  Greedy outputs must equal a single engine's."""
import multiprocessing as mp
import os
import socket

import pytest

from tests._tiny import random_prompts, tiny_llama_checkpoint

MAX_TOKENS = [9, 4, 12, 1]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, ckpt, prompts, prefill_tokens, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch

    torch.set_num_threads(1)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    try:
        role = "kv_producer" if rank == 0 else "kv_consumer"
        llm = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
                  max_num_batched_tokens=64, kv_transfer_config={"kv_role": role})
        if rank == 0:
            outs = llm.generate(prompts, [SamplingParams(temperature=0, max_tokens=min(prefill_tokens, n),
                                                         ignore_eos=True) for n in MAX_TOKENS])
            q.put((rank, ([o.outputs[0].token_ids for o in outs], llm.engine.kv_connector.sent)))
        else:
            # the decode parameters of each request, by request id (as a routing proxy would)
            params = lambda rid: SamplingParams(temperature=0, max_tokens=MAX_TOKENS[int(rid.rsplit("-", 1)[1])],
                                                ignore_eos=True)
            outs = llm.generate_remote(len(prompts), params)
            q.put((rank, ({o.request_id: o.outputs[0].token_ids for o in outs}, llm.engine.kv_connector.bytes)))
    except Exception:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        ps.destroy_parallel_state()


@pytest.mark.parametrize("prefill_tokens", [1, 3])
def test_prefill_decode_handoff_matches_single_engine(prefill_tokens):
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ckpt, _ = tiny_llama_checkpoint()
    prompts = [p[:n] for p, n in zip(random_prompts(n=4, length=40, seed=5), (40, 17, 33, 8))]
    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=64).generate(
        prompts, [SamplingParams(temperature=0, max_tokens=n, ignore_eos=True) for n in MAX_TOKENS])
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, ckpt, prompts, prefill_tokens, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in (1, 0):  # a consumer failure also breaks the producer's send
        assert not isinstance(res[r], str), res[r]
    pre, sent = res[0]
    assert sent == len(prompts)
    assert pre == [r[:min(prefill_tokens, n)] for r, n in zip(ref, MAX_TOKENS)]
    by_id, nbytes = res[1]
    assert nbytes > 0
    got = [by_id[k] for k in sorted(by_id, key=lambda s: int(s.rsplit("-", 1)[1]))]
    assert got == ref, (got, ref)
