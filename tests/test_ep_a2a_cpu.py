"""Expert parallelism with all-to-all token exchange on CPU: the dispatch metadata / packing /
top-k reduction ops, the exchange over two gloo ranks holding different tokens, and two
data-parallel replicas of a Qwen3-MoE model serving in lockstep with experts sharded across
them (greedy tokens equal a single-process run)."""
import multiprocessing as mp
import os
import socket
import tempfile

import torch

from tests._tiny import random_prompts
from vllm_neuron_b200.ops import ep as EP
from vllm_neuron_b200.ops import moe as M


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(E, H, I, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(E, 2 * I, H, generator=g) * 0.1, torch.randn(E, H, I, generator=g) * 0.1


def test_dispatch_metadata_dedups_tokens_per_rank():
    ids = torch.tensor([[0, 1], [2, 5], [4, 5], [7, 6]], dtype=torch.int32)  # e_local = 2, 4 ranks
    plan, hit = EP.build_dispatch_metadata(ids, e_local=2, world=4)
    assert plan.send_counts == [1, 1, 2, 1]          # token 0's two experts share rank 0
    assert plan.dest_of_row.tolist() == [0, 1, 2, 2, 3]
    assert plan.token_of_row.tolist() == [0, 1, 1, 2, 3]
    x = torch.arange(4.0)[:, None].repeat(1, 3)
    w = torch.tensor([[0.6, 0.4], [0.7, 0.3], [0.5, 0.5], [0.9, 0.1]])
    rows, aff = EP.permute_routed_tokens(x, ids, w, plan, e_local=2)
    assert rows[:, 0].tolist() == [0, 1, 1, 2, 3]
    assert torch.allclose(aff, torch.tensor([[0.6, 0.4], [0.7, 0.0], [0.0, 0.3], [0.5, 0.5], [0.1, 0.9]]))
    assert EP.pack_tokens(torch.tensor([-1, 3, -1, 0])).tolist() == [1, 3]


def test_single_rank_roundtrip_equals_moe_block():
    from vllm_neuron_b200.parallel.all2all import All2AllManager

    E, H, I, T, k = 8, 32, 16, 11, 3
    w_gu, w_down = _weights(E, H, I)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(T, H, generator=g)
    router = torch.randn(E, H, generator=g)
    ref = M.moe_block(x, router, w_gu, w_down, k, M.ROUTE_SOFTMAX_TOPK, True, out=torch.empty(T, H))
    logits = (x @ router.t())
    ids, w = M.route(logits, k, M.ROUTE_SOFTMAX_TOPK, True)
    a2a = All2AllManager(None, 0, 1, E)
    plan, rows, aff = a2a.dispatch(x, ids, w)
    lids, lw = EP.local_routing(aff, 0, k)
    part = M.moe_experts(rows, lids, lw, w_gu, w_down)
    out = a2a.combine(part, plan)
    assert torch.allclose(out.float(), ref.float(), atol=1e-4)


def _exchange_worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    import torch.distributed as dist

    torch.set_num_threads(1)
    from vllm_neuron_b200.parallel.all2all import All2AllManager

    try:
        dist.init_process_group("gloo")
        E, H, I, k = 8, 32, 16, 3
        w_gu, w_down = _weights(E, H, I)                    # same full weights on both ranks
        g = torch.Generator().manual_seed(10 + rank)        # different tokens per rank
        T = 9 if rank == 0 else 4
        x = torch.randn(T, H, generator=g)
        ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
        w = torch.rand(T, k, generator=g)
        a2a = All2AllManager(dist.group.WORLD, rank, 2, E)
        plan, rows, aff = a2a.dispatch(x, ids, w)
        lids, lw = EP.local_routing(aff, a2a.e_start, k)
        el = a2a.e_local
        part = M.moe_experts(rows, lids, lw, w_gu[a2a.e_start:a2a.e_start + el],
                             w_down[a2a.e_start:a2a.e_start + el], e_start=a2a.e_start)
        out = a2a.combine(part, plan)
        ref = M.experts_ref(x, ids, w, w_gu, w_down)
        q.put((rank, float((out.float() - ref).abs().max())))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def _run(target, *args, n=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=target, args=(r, port) + args + (q,)) for r in range(n)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    return res


def test_two_rank_exchange_matches_all_experts():
    res = _run(_exchange_worker)
    for r in (0, 1):
        assert isinstance(res[r], float) and res[r] < 1e-4, res


def _qwen_moe_ckpt():
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    torch.manual_seed(1)
    cfg = Qwen3MoeConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=16, intermediate_size=128, moe_intermediate_size=32, num_experts=8,
                         num_experts_per_tok=2, norm_topk_prob=True, vocab_size=512,
                         max_position_embeddings=256, initializer_range=0.05)
    hf = Qwen3MoeForCausalLM(cfg).float().eval()
    d = tempfile.mkdtemp(prefix="tiny_qwen_moe_ep_")
    hf.save_pretrained(d, safe_serialization=True)
    return d


_KW = dict(device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
           max_num_batched_tokens=64)


def _dp_worker(rank, port, ckpt, prompts, e_local, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    try:
        llm = LLM(ckpt, data_parallel_size=2, enable_expert_parallel=True,
                  additional_config={"neuron_config": {"all2all_backend": "nccl"}}, **_KW)
        m = llm.engine.model
        assert m.a2a is not None and m.e_local == e_local and m.e_start == e_local * rank
        outs = llm.generate(prompts, [SamplingParams(temperature=0, max_tokens=n, ignore_eos=True)
                                      for n in (8, 3, 12, 5, 1)])
        q.put((rank, ([o.outputs[0].token_ids for o in outs], m.a2a.calls)))
    except Exception as e:  # pragma: no cover
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        ps.destroy_parallel_state()


def test_dp2_wide_ep_lockstep_matches_single_process():
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ckpt = _qwen_moe_ckpt()
    prompts = [p[:n] for p, n in zip(random_prompts(n=5, length=30, vocab=512, seed=3), (30, 7, 19, 25, 4))]
    ref = LLM(ckpt, **_KW).generate(prompts, [SamplingParams(temperature=0, max_tokens=n, ignore_eos=True)
                                             for n in (8, 3, 12, 5, 1)])
    ref = [o.outputs[0].token_ids for o in ref]
    res = _run(_dp_worker, ckpt, prompts, 4)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
        toks, calls = res[r]
        assert toks == ref, (r, toks, ref)
        assert calls > 0


def test_dp2_wide_ep_gpt_oss():
    """GPT-OSS (biased experts, clamped SwiGLU, top-k-then-softmax routing) with its experts
    split over two data-parallel replicas by all-to-all."""
    from tests.test_gpt_oss_cpu import _tiny_gpt_oss
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ckpt, _ = _tiny_gpt_oss()
    prompts = [p[:n] for p, n in zip(random_prompts(n=5, length=30, vocab=512, seed=4), (30, 7, 19, 25, 4))]
    ref = LLM(ckpt, **_KW).generate(prompts, [SamplingParams(temperature=0, max_tokens=n, ignore_eos=True)
                                             for n in (8, 3, 12, 5, 1)])
    ref = [o.outputs[0].token_ids for o in ref]
    res = _run(_dp_worker, ckpt, prompts, 2)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
        assert res[r][0] == ref, (r, res[r][0], ref)
