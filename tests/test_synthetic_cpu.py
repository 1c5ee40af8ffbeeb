"""KV-cache plumbing through the synthetic model: every emitted status token must be 5 (all KV
read back through the block tables matches what was written), under chunked prefill, prefix
caching and preemption."""
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM

CFG = {"architectures": ["SyntheticForCausalLM"], "model_type": "synthetic", "hidden_size": 64,
       "num_hidden_layers": 3, "num_attention_heads": 2, "num_key_value_heads": 2, "head_dim": 16,
       "vocab_size": 16, "max_position_embeddings": 512}


def _run(**kw):
    prompts = [[1] * 40, [2] * 75, [1] * 40 + [3] * 10, [4] * 9]
    llm = LLM(dict(CFG), device="cpu", dtype="float32", max_num_seqs=4, max_model_len=256,
              load_format="dummy", skip_tokenizer_init=True, **kw)
    outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=20, ignore_eos=True))
    return [o.outputs[0].token_ids for o in outs]


def test_kv_roundtrip_chunked_prefix_and_preemption():
    for kw in (dict(num_gpu_blocks=64, max_num_batched_tokens=256),
               dict(num_gpu_blocks=64, max_num_batched_tokens=16),
               dict(num_gpu_blocks=64, max_num_batched_tokens=64, enable_prefix_caching=True),
               dict(num_gpu_blocks=14, max_num_batched_tokens=32)):  # forces preemption
        outs = _run(**kw)
        assert all(t == 5 for o in outs for t in o), (kw, outs)
