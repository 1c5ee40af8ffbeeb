"""Structured outputs on CPU: with a grammar, every generated token sequence must match it
(regex / choice / JSON schema), whatever the random model prefers; other requests in the same
batch are unaffected."""
import json
import re

import torch

from tests._tiny import random_prompts, tiny_llama_checkpoint
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM
from vllm_neuron_b200.ops.sampling import apply_token_bitmask

V = 32000
EOS = 31999


def _vocab():
    # a synthetic byte-level vocabulary: printable characters first, other ids are opaque
    chars = [chr(c) for c in range(32, 127)]
    vocab = chars + [f"<t{i}>" for i in range(len(chars), V)]
    vocab[EOS] = "</s>"
    return vocab


def _llm():
    d, _ = tiny_llama_checkpoint()
    llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=64)
    llm.engine.eos_token_id = EOS
    llm.engine.structured_vocab = _vocab()
    return llm


def _text(ids):
    v = _vocab()
    return "".join(v[i] for i in ids if i != EOS)


def test_bitmask_ref():
    logits = torch.zeros(2, 40)
    mask = torch.tensor([[0b101, 0], [-1, -1]], dtype=torch.int32)
    apply_token_bitmask(logits, mask)
    assert torch.isfinite(logits[0]).nonzero().flatten().tolist() == [0, 2]
    assert torch.isfinite(logits[1]).all()


def test_regex_choice_json():
    llm = _llm()
    prompts = random_prompts(n=4, length=10)
    sps = [SamplingParams(temperature=0, max_tokens=20, structured_outputs={"regex": "ab(1|2)[xyz]{2}"}),
           SamplingParams(temperature=0.8, seed=1, max_tokens=20, structured_outputs={"choice": ["yes", "no"]}),
           SamplingParams(temperature=0, max_tokens=60, structured_outputs={"json": {
               "type": "object", "properties": {"a": {"type": "integer"}}, "required": ["a"]}}),
           SamplingParams(temperature=0, max_tokens=5, ignore_eos=True)]
    outs = llm.generate(prompts, sps)
    assert re.fullmatch("ab(1|2)[xyz]{2}", _text(outs[0].outputs[0].token_ids))
    assert _text(outs[1].outputs[0].token_ids) in ("yes", "no")
    obj = json.loads(_text(outs[2].outputs[0].token_ids))
    assert isinstance(obj["a"], int)
    assert len(outs[3].outputs[0].token_ids) == 5
