"""Aux subsystems on CPU: logit validation against HF, three-way closeness, hidden-state
capture, snapshot capture of step inputs, profiler traces."""
import os

import pytest
import torch

from tests._tiny import random_prompts, tiny_llama_checkpoint
from vllm_neuron_b200.accuracy import assert_close_three_way, capture_hidden, compare_logits, validate_against_hf
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM

KW = dict(device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=32,
          max_num_batched_tokens=128)


def test_logit_validation_and_capture():
    d, hf = tiny_llama_checkpoint()
    llm = LLM(d, **KW)
    prompts = random_prompts(n=2, length=12)
    rep = validate_against_hf(llm.engine, hf, prompts)
    assert rep.passed(rel_tol=1e-4, min_argmax=1.0) and rep.kl_div < 1e-6
    h = capture_hidden(llm.engine, prompts, [0, 1])
    with torch.no_grad():
        hs = hf(torch.tensor([prompts[0]]), output_hidden_states=True).hidden_states
    assert torch.allclose(h[:12, 0], hs[1][0], atol=1e-4)


def test_three_way():
    o = torch.randn(100)
    lo = o + 1e-2 * torch.randn(100)
    assert_close_three_way(o, lo, o + 1e-2 * torch.randn(100))
    with pytest.raises(AssertionError):
        assert_close_three_way(o, lo, o + 1.0)
    r = compare_logits(torch.randn(3, 50), torch.randn(3, 50))
    assert 0 <= r.topk_overlap <= 1


def test_snapshot_and_profile(tmp_path, monkeypatch):
    monkeypatch.setenv("VLLM_B200_SNAPSHOT_DIR", str(tmp_path / "snap"))
    d, _ = tiny_llama_checkpoint()
    llm = LLM(d, **KW)
    llm.engine.start_profile(str(tmp_path / "prof"))
    llm.generate(random_prompts(n=2, length=8), SamplingParams(temperature=0, max_tokens=3, ignore_eos=True))
    path = llm.engine.stop_profile()
    assert path and os.path.getsize(path) > 0
    snaps = sorted(os.listdir(tmp_path / "snap"))
    assert len(snaps) >= 3
    s0 = torch.load(tmp_path / "snap" / snaps[0])
    assert s0["layout"]["T"] == 16 and len(s0["requests"]) == 2
