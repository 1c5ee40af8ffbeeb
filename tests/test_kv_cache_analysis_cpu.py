"""KV-cache analysis on the CPU: the framework's paged KV for a prompt, gathered back into
contiguous tensors, against the teacher-forced Hugging Face KV of the same checkpoint.

* fp32 engine vs fp32 HF: cosine ~1 and relative errors at fp32 rounding for every (layer,
  head, token).
* fp8 KV cache: the same comparison shows the e4m3 quantization (relative L2 around 2-6 %),
  and the three-way form (expected = fp32 HF, baseline = HF, actual = fp8 engine) reports
  low error-distribution agreement against the fp32 engine's.
"""
import numpy as np
import torch

from tests._tiny import random_prompts, tiny_llama_checkpoint
from vllm_neuron_b200.accuracy import kv_cache_analysis as KA
from vllm_neuron_b200.entrypoints import LLM


def _llm(ckpt, **kw):
    return LLM(ckpt, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
               max_num_batched_tokens=64, **kw)


def test_engine_kv_matches_hf():
    ckpt, hf = tiny_llama_checkpoint()
    prompt = random_prompts(n=1, length=45, seed=3)[0]
    exp = KA.hf_kv(hf, prompt)
    act = KA.extract_request_kv(_llm(ckpt), prompt)
    assert act.k.shape == exp.k.shape and act.num_tokens == 45
    cmp = KA.compare_kv_caches(exp, act)
    s = cmp.summary()
    assert s["k_cos_min"] > 0.99999 and s["v_cos_min"] > 0.99999, s
    assert s["k_l2_max"] < 1e-4 and s["v_l2_max"] < 1e-4, s
    rep = KA.format_kv_report(cmp)
    assert "KV cache comparison" in rep and "worst K" in rep


def test_fp8_cache_three_way():
    ckpt, hf = tiny_llama_checkpoint()
    prompt = random_prompts(n=1, length=40, seed=4)[0]
    base = KA.hf_kv(hf, prompt)
    exact = KA.extract_request_kv(_llm(ckpt), prompt)
    fp8 = KA.extract_request_kv(_llm(ckpt, kv_cache_dtype="fp8"), prompt)
    plain = KA.compare_kv_caches(base, fp8)
    s = plain.summary()
    assert 0.95 < s["k_cos_min"] < 0.99999, s  # e4m3 rounding is visible, nothing is broken
    assert 1e-3 < s["k_l2_max"] < 0.2, s
    # three-way: the fp32 engine errs like the reference (BC ~1); the fp8 engine does not
    same = KA.compare_kv_caches(exact, exact, baseline=base)
    diff = KA.compare_kv_caches(exact, fp8, baseline=base)
    assert min(same.token_bc_k) > 0.99
    assert np.mean(diff.token_bc_k) < np.mean(same.token_bc_k)
    assert len(diff.token_bc_k) == 40
    w = diff.worst("k", "l2", top=3)
    assert len(w) == 3 and all(0 <= l < base.k.shape[0] for l, _, _, _ in w)


def test_bhattacharyya():
    a = np.random.default_rng(0).normal(size=5000)
    assert KA.bhattacharyya(a, a) > 0.999
    assert KA.bhattacharyya(a, a + 10.0) < 0.05
    assert KA.bhattacharyya(np.zeros(10), np.zeros(10)) == 1.0
