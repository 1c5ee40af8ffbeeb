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
    snaps = sorted(f for f in os.listdir(tmp_path / "snap") if f.endswith(".pt"))
    assert len(snaps) >= 3
    s0 = torch.load(tmp_path / "snap" / snaps[0])
    assert s0["layout"]["T"] == 16 and len(s0["requests"]) == 2
    assert os.path.exists(tmp_path / "snap" / snaps[0].replace(".pt", ".meta.json"))


def test_snapshot_selection_and_replay(tmp_path, monkeypatch):
    """Step selection rules, and a captured prefill step replayed through the runner gives the
    logits of the original run."""
    from vllm_neuron_b200.snapshot import load_snapshot, replay_logits
    from vllm_neuron_b200.snapshot.config import SnapshotConfig, parse_index_set

    assert parse_index_set("0,3-5", "x") == (False, {0, 3, 4, 5})
    assert parse_index_set("all", "x") == (True, None)
    import pytest as _pt

    with _pt.raises(ValueError):
        parse_index_set("3-1", "x")
    cfg = SnapshotConfig.from_env({"VLLM_B200_SNAPSHOT_DIR": "/x", "VLLM_B200_SNAPSHOT_TOKENS": "9",
                                   "VLLM_B200_SNAPSHOT_REQUESTS": "r1"})
    assert cfg.selector.matches(5, [(0, 8)], ["r1"]) and cfg.selector.matches(5, [(8, 10)], ["r0"])
    assert not cfg.selector.matches(5, [(0, 8)], ["r0"])
    d, _ = tiny_llama_checkpoint()
    monkeypatch.setenv("VLLM_B200_SNAPSHOT_DIR", str(tmp_path / "snap"))
    monkeypatch.setenv("VLLM_B200_SNAPSHOT_AT_STEP", "0")
    llm = LLM(d, **KW)
    prompts = random_prompts(n=2, length=8)
    ref = llm.engine.prompt_logits(prompts)  # step 0: a prefill from an empty cache
    files = sorted(f for f in os.listdir(tmp_path / "snap") if f.endswith(".pt"))
    assert len(files) == 1
    snap = load_snapshot(str(tmp_path / "snap" / files[0]))
    got = replay_logits(llm.engine.runner, snap)
    assert torch.allclose(got.float(), ref[:, :got.shape[1]], atol=1e-5)
