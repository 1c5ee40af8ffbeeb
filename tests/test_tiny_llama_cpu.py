"""Plumbing config: tiny Llama-3 on CPU (fp32), greedy decode of 16 tokens for 4 prompts of
32 random tokens through LLM.generate with paged KV block size 16; must match HF exactly."""
import torch

from tests._tiny import random_prompts, tiny_llama_checkpoint
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM


def _hf_greedy(hf, prompt, n):
    ids = torch.tensor([prompt])
    out = []
    with torch.no_grad():
        for _ in range(n):
            nxt = int(hf(ids).logits[0, -1].argmax())
            out.append(nxt)
            ids = torch.cat([ids, torch.tensor([[nxt]])], 1)
    return out


def test_tiny_llama_generate_matches_hf():
    d, hf = tiny_llama_checkpoint()
    prompts = random_prompts()
    llm = LLM(d, device="cpu", max_num_seqs=8, max_model_len=256, num_gpu_blocks=64, block_size=16,
              max_num_batched_tokens=64)
    outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=16, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert o.outputs[0].token_ids == _hf_greedy(hf, p, 16)
        assert o.outputs[0].finish_reason == "length"


def test_chunked_prefill_and_prefix_cache_consistent():
    d, hf = tiny_llama_checkpoint()
    prompts = random_prompts(n=3, length=70, seed=3)
    sp = SamplingParams(temperature=0, max_tokens=5, ignore_eos=True)
    base = LLM(d, device="cpu", max_num_seqs=4, max_model_len=256, num_gpu_blocks=64,
               max_num_batched_tokens=256).generate(prompts, sp)
    chunked = LLM(d, device="cpu", max_num_seqs=4, max_model_len=256, num_gpu_blocks=64,
                  max_num_batched_tokens=24).generate(prompts, sp)
    llm = LLM(d, device="cpu", max_num_seqs=4, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=256, enable_prefix_caching=True)
    first = llm.generate(prompts, sp)
    second = llm.generate(prompts, sp)
    for a, b, c, e in zip(base, chunked, first, second):
        assert a.outputs[0].token_ids == b.outputs[0].token_ids == c.outputs[0].token_ids == e.outputs[0].token_ids
    assert any(o.metrics["num_cached_tokens"] > 0 for o in second)


def test_preemption_under_block_pressure():
    d, hf = tiny_llama_checkpoint()
    prompts = random_prompts(n=6, length=40, seed=5)
    sp = SamplingParams(temperature=0, max_tokens=20, ignore_eos=True)
    ref = LLM(d, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64).generate(prompts, sp)
    # 13 usable blocks cannot hold six 60-token sequences at once -> preemption + recompute
    tight = LLM(d, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=14)
    outs = tight.generate(prompts, sp)
    assert [o.outputs[0].token_ids for o in outs] == [o.outputs[0].token_ids for o in ref]


def test_async_scheduling_matches_sync():
    """Asynchronous scheduling (step N+1 launched before step N's tokens are processed; decode
    inputs read from the device-resident token slots) yields the same tokens, including when a
    stop token ends a request while its next step is already in flight."""
    d, hf = tiny_llama_checkpoint()
    prompts = random_prompts(n=5, length=24, seed=7)
    kw = dict(device="cpu", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64, max_num_batched_tokens=40)
    sync = LLM(d, async_scheduling=False, **kw)
    base = sync.generate(prompts, SamplingParams(temperature=0, max_tokens=12, ignore_eos=True))
    stop_tok = base[1].outputs[0].token_ids[4]
    sps = [SamplingParams(temperature=0, max_tokens=12, ignore_eos=True)] * 5
    sps[1] = SamplingParams(temperature=0, max_tokens=12, stop_token_ids=[stop_tok])
    ref = sync.generate(prompts, sps)
    asy = LLM(d, async_scheduling=True, **kw)
    got = asy.generate(prompts, sps)
    assert [o.outputs[0].token_ids for o in got] == [o.outputs[0].token_ids for o in ref]
    assert got[1].outputs[0].finish_reason == "stop"
    assert len(asy.engine._free_slots) == asy.engine.runner.max_slots - 1


def test_prompt_embeds_match_token_prompts():
    """Passing the embedding rows of a prompt instead of its ids gives the same generation."""
    d, hf = tiny_llama_checkpoint()
    prompts = random_prompts(n=2, length=20)
    sp = SamplingParams(temperature=0, max_tokens=6, ignore_eos=True)
    llm = LLM(d, device="cpu", max_num_seqs=4, max_model_len=128, num_gpu_blocks=32, max_num_batched_tokens=16)
    ref = llm.generate(prompts, sp)
    emb = hf.get_input_embeddings().weight.detach()
    got = llm.generate([{"prompt_embeds": emb[torch.tensor(p)]} for p in prompts], sp)
    assert [o.outputs[0].token_ids for o in got] == [o.outputs[0].token_ids for o in ref]
