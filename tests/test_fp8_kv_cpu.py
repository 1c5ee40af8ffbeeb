"""FP8 KV cache on the CPU path: quantization rule, oracle dequantization, engine plumbing
(cache dtype, block bytes, checkpoint scales) and generation through ``LLM``."""
import numpy as np
import torch

from vllm_neuron_b200 import ops
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM

CFG = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 256,
       "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
       "intermediate_size": 512, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
       "max_position_embeddings": 1024}


def test_quantize_rule_saturates_and_rounds():
    x = torch.tensor([0.0, 1.0, -3.3, 1000.0, -1e6, 0.013])
    q = ops.attention.quantize_kv_fp8(x, 0.5)
    assert q.dtype == torch.float8_e4m3fn
    back = q.float() * 0.5
    assert back[3].item() == 448.0 * 0.5 and back[4].item() == -448.0 * 0.5  # saturated
    assert abs(back[2].item() + 3.3) / 3.3 < 1 / 16 + 1e-6                    # 3 mantissa bits
    assert back[0].item() == 0.0


def test_oracle_dequantizes_with_scales():
    g = torch.Generator().manual_seed(0)
    Hq, Hkv, D, bs, nb = 4, 2, 64, 16, 6
    k = torch.randn(nb, Hkv, bs, D, generator=g)
    v = torch.randn(nb, Hkv, bs, D, generator=g)
    ks, vs = 0.03, 0.01
    k8, v8 = ops.attention.quantize_kv_fp8(k, ks), ops.attention.quantize_kv_fp8(v, vs)
    q = torch.randn(3, Hq, D, generator=g)
    bt = torch.tensor([[1, 2, 3, 4]], dtype=torch.int32)
    sl = torch.tensor([50], dtype=torch.int32)
    qs = torch.tensor([0, 3], dtype=torch.int32)
    got = ops.paged_attention_ref(q, k8, v8, bt, sl, qs, 0.125, k_scale=ks, v_scale=vs)
    want = ops.paged_attention_ref(q, k8.float() * ks, v8.float() * vs, bt, sl, qs, 0.125)
    assert torch.allclose(got, want, atol=1e-5)
    exact = ops.paged_attention_ref(q, k, v, bt, sl, qs, 0.125)
    assert ((got - exact).norm() / exact.norm()).item() < 0.1


def test_llm_fp8_cache_generates_like_full_precision():
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 32000, (32,), generator=g).tolist() for _ in range(4)]
    toks, logits = {}, {}
    for kv in ("auto", "fp8"):
        llm = LLM(CFG, max_num_seqs=4, max_model_len=256, num_gpu_blocks=64, load_format="dummy",
                  device="cpu", skip_tokenizer_init=True, kv_cache_dtype=kv)
        r = llm.engine.runner
        if kv == "fp8":
            assert r.kv_cache.dtype == torch.float8_e4m3fn
            assert r.kv_bytes_per_block() * 4 == bytes_auto  # fp32 CPU model -> 1-byte cache
        else:
            bytes_auto = r.kv_bytes_per_block()
        logits[kv] = llm.engine.prompt_logits(prompts)
        outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
        toks[kv] = [o.outputs[0].token_ids for o in outs]
        llm.shutdown()
    err = ((logits["fp8"] - logits["auto"]).norm() / logits["auto"].norm()).item()
    assert err < 5e-2
    assert sum(a[0] == b[0] for a, b in zip(toks["fp8"], toks["auto"])) >= 3


def test_kv_scales_read_from_checkpoint(tmp_path):
    from safetensors.torch import save_file

    from vllm_neuron_b200.engine.llm_engine import _kv_scales_from_checkpoint

    save_file({"model.layers.0.self_attn.k_scale": torch.tensor(0.25),
               "model.layers.1.self_attn.v_scale": torch.tensor([0.5])},
              str(tmp_path / "model.safetensors"))

    class M:
        num_kv_layers = 2

    assert _kv_scales_from_checkpoint(M(), str(tmp_path)) == [(0.25, 1.0), (1.0, 0.5)]
    assert _kv_scales_from_checkpoint(M(), None) is None


def test_rejects_unknown_kv_dtype():
    import pytest

    with pytest.raises(ValueError):
        LLM(CFG, max_num_seqs=2, max_model_len=64, num_gpu_blocks=16, load_format="dummy",
            device="cpu", skip_tokenizer_init=True, kv_cache_dtype="int4")
