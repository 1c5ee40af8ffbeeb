"""Activation capture, golden replacement and capture comparison (accuracy tooling) on CPU.

* The per-layer residual captures of a generation equal HF's ``hidden_states`` at every prompt
  position, and do not depend on how the prompt was chunked.
* Replacing layer 0's output with a reference run's rows makes a model with different layer-0
  weights reproduce the reference from layer 1 on; without it the comparison localises the
  divergence at layer 0.
"""
import torch

from tests._tiny import random_prompts, tiny_llama_checkpoint
from vllm_neuron_b200.accuracy import compare_captures, expand_patterns, first_divergence, format_report
from vllm_neuron_b200.accuracy.tensor_compare import load_dir
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM


def _llm(d, chunk=256, **opts):
    return LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
               max_num_batched_tokens=chunk, additional_config={"b200_config": opts} if opts else None)


def test_expand_patterns():
    assert expand_patterns(["model.layers.0-2", "lm_head"]) == [
        "model.layers.0", "model.layers.1", "model.layers.2", "lm_head"]
    assert expand_patterns(["model.layers.1-2.x"]) == ["model.layers.1.x", "model.layers.2.x"]


def test_capture_matches_hf_hidden_states_and_ignores_chunking(tmp_path):
    d, hf = tiny_llama_checkpoint()
    prompts = random_prompts(n=2, length=24)
    sp = SamplingParams(temperature=0, max_tokens=3, ignore_eos=True)
    caps = {}
    for chunk in (256, 8):
        out = tmp_path / f"cap{chunk}"
        llm = _llm(d, chunk, tensor_capture={"modules": ["model.layers.0-1", "model.norm", "lm_head"],
                                             "capture_dir": str(out)})
        assert not llm.engine.runner.use_graphs
        llm.generate(prompts, sp)
        caps[chunk] = load_dir(str(out))
    a, b = caps[256], caps[8]
    assert set(a) == set(b) and len(a) == 2
    for key in a:
        for name in ("model.layers.0", "model.layers.1", "model.norm", "lm_head"):
            assert torch.allclose(a[key][name], b[key][name], atol=1e-4), name
        # 24 prompt positions + 2 decoded positions (the 3rd token is never fed back)
        assert a[key]["model.layers.0"].shape[0] == 26
        assert a[key]["lm_head"].shape[0] == 3
        with torch.no_grad():
            hs = hf(torch.tensor([list(key)]), output_hidden_states=True).hidden_states
        for i in range(2):
            got = a[key][f"model.layers.{i}"][:24]
            ref = hs[i + 1][0] if i + 1 < len(hs) - 1 else None
            if ref is not None:  # HF's last entry is after the final norm
                assert torch.allclose(got, ref, atol=2e-4), i
        assert torch.allclose(a[key]["model.norm"][:24], hs[-1][0], atol=2e-4)


def test_replacement_pins_layer_and_compare_localises(tmp_path):
    d, _ = tiny_llama_checkpoint()
    prompts = random_prompts(n=2, length=16, seed=3)
    sp = SamplingParams(temperature=0, max_tokens=1, ignore_eos=True)
    mods = ["model.layers.0-1", "lm_head"]
    gold = tmp_path / "gold"
    _llm(d, tensor_capture={"modules": mods, "capture_dir": str(gold)}).generate(prompts, sp)

    def perturbed(**opts):
        llm = _llm(d, **opts)
        with torch.no_grad():  # a different layer 0 (its MLP down projection)
            w = llm.engine.model.layers[0].down
            w.add_(0.05 * torch.randn(w.shape, generator=torch.Generator().manual_seed(1)))
        return llm

    bad = tmp_path / "bad"
    perturbed(tensor_capture={"modules": mods, "capture_dir": str(bad)}).generate(prompts, sp)
    rep = compare_captures(str(gold), str(bad))
    first = first_divergence(rep, rel_tol=1e-3)
    assert first is not None and first.point == "model.layers.0", format_report(rep)

    fixed = tmp_path / "fixed"
    llm = perturbed(tensor_capture={"modules": mods, "capture_dir": str(fixed)},
                    tensor_replacement={"golden_dir": str(gold), "modules": ["model.layers.0"]})
    llm.generate(prompts, sp)
    assert llm.engine.model.capture.replace.replaced == 2 * 16
    rep = compare_captures(str(gold), str(fixed))
    assert first_divergence(rep, rel_tol=1e-4) is None, format_report(rep)
