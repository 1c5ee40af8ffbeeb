"""Speculative decoding on CPU: whatever the proposer drafts, greedy output must equal plain
greedy decoding (the target model verifies every token); the n-gram proposer and the
rejection sampler are checked against small oracles."""
import torch

from tests._tiny import random_prompts, tiny_llama_checkpoint
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM
from vllm_neuron_b200.spec_decode import NgramProposer, rejection_sample, rejection_sample_ref


def test_ngram_proposer():
    p = NgramProposer(3, 1, 3)
    assert p.propose_one([1, 2, 3, 9, 1, 2, 3]) == [9, 1, 2]
    assert p.propose_one([5, 6, 7]) == []
    assert p.propose_one([4, 4, 4, 4]) == [4]


def test_rejection_sampler_greedy_matches_oracle():
    torch.manual_seed(0)
    drafts = [[3, 1, 4], [2], [], [7, 7]]
    n = sum(len(d) + 1 for d in drafts)
    logits = torch.randn(n, 10)
    am = logits.argmax(-1).tolist()
    # force some acceptances
    logits[0, 3] = 10
    logits[1, 1] = 10
    am = logits.argmax(-1).tolist()
    rows, r = [], 0
    for d in drafts:
        rows.append(am[r:r + len(d) + 1])
        r += len(d) + 1
    got = rejection_sample(logits, drafts, [0.0] * 4)
    assert got == rejection_sample_ref(rows, drafts)
    assert got[0][:2] == [3, 1]


def test_rejection_sampler_random_keeps_target_distribution():
    # one draft token, target p over 4 tokens: P(output = t) must equal p(t)
    p = torch.tensor([0.1, 0.2, 0.3, 0.4])
    logits = torch.log(p).repeat(2, 1)
    g = torch.Generator().manual_seed(0)
    counts = torch.zeros(4)
    for _ in range(4000):
        counts[rejection_sample(logits, [[2]], [1.0], [g])[0][0]] += 1
    assert torch.allclose(counts / counts.sum(), p, atol=0.03)


def test_ngram_spec_decode_matches_greedy():
    d, _ = tiny_llama_checkpoint()
    # prompts with repetition so the n-gram proposer finds drafts
    base = random_prompts(n=3, length=12)
    prompts = [b + b + b[:6] for b in base]
    sp = SamplingParams(temperature=0, max_tokens=16, ignore_eos=True)
    kw = dict(device="cpu", dtype="float32", max_num_seqs=4, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=64)
    ref = LLM(d, **kw).generate(prompts, sp)
    llm = LLM(d, speculative_config={"method": "ngram", "num_speculative_tokens": 3}, **kw)
    got = llm.generate(prompts, sp)
    assert [o.outputs[0].token_ids for o in got] == [o.outputs[0].token_ids for o in ref]
    m = llm.engine.metrics
    assert m.spec_draft_tokens > 0


def test_eagle3_spec_decode_matches_greedy(tmp_path):
    """An EAGLE3 draft head (random weights, saved in the checkpoint layout and loaded back)
    proposes; output must equal plain greedy decoding."""
    from safetensors.torch import save_file

    d, _ = tiny_llama_checkpoint()
    H, Hq, Hkv, D, I, V = 256, 4, 2, 64, 512, 32000
    g = torch.Generator().manual_seed(3)
    r = lambda *s: torch.randn(*s, generator=g) * 0.05  # noqa: E731
    t = {"fc.weight": r(H, 3 * H), "norm.weight": torch.ones(H), "lm_head.weight": r(V, H),
         "d2t": torch.zeros(V, dtype=torch.int64)}
    for n, shape in (("self_attn.q_proj.weight", (Hq * D, 2 * H)), ("self_attn.k_proj.weight", (Hkv * D, 2 * H)),
                     ("self_attn.v_proj.weight", (Hkv * D, 2 * H)), ("self_attn.o_proj.weight", (H, Hq * D)),
                     ("mlp.gate_proj.weight", (I, H)), ("mlp.up_proj.weight", (I, H)), ("mlp.down_proj.weight", (H, I))):
        t["midlayer." + n] = r(*shape)
    for n in ("input_layernorm", "hidden_norm", "post_attention_layernorm"):
        t[f"midlayer.{n}.weight"] = torch.ones(H)
    save_file(t, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text('{"architectures": ["LlamaForCausalLMEagle3"], "intermediate_size": 512}')
    prompts = random_prompts(n=2, length=20)
    sp = SamplingParams(temperature=0, max_tokens=12, ignore_eos=True)
    kw = dict(device="cpu", dtype="float32", max_num_seqs=4, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=64)
    ref = LLM(d, **kw).generate(prompts, sp)
    llm = LLM(d, speculative_config={"method": "eagle3", "num_speculative_tokens": 3, "model": str(tmp_path),
                                     "aux_layers": [0, 1, 1]}, **kw)
    got = llm.generate(prompts, sp)
    assert [o.outputs[0].token_ids for o in got] == [o.outputs[0].token_ids for o in ref]
    assert llm.engine.metrics.spec_draft_tokens > 0
