"""Host-side units: config parsing, block manager, scheduler policy, group rank math."""
import pytest
import torch

from vllm_neuron_b200.config import B200Config, ModelArchConfig
from vllm_neuron_b200.engine.block_manager import BlockManager
from vllm_neuron_b200.engine.request import Request
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.engine.scheduler import Scheduler, bucket_for
from vllm_neuron_b200.parallel import state as ps


def test_b200_config_accepts_reference_keys():
    c = B200Config.from_additional_config({"neuron_config": {
        "ep_degree": 8, "attention_dp_size": 2, "num_batched_tokens_buckets": [512, 128, 256],
        "on_device_sampling_config": {"global_topk": 64}, "quantization": "fp8", "unknown_key": 1}})
    assert c.ep_degree == 8 and c.attention_dp_size == 2
    assert c.num_batched_tokens_buckets == [128, 256, 512]
    assert c.on_device_sampling_config.global_topk == 64 and c.on_device_sampling_config.enabled
    assert c.extra == {"unknown_key": 1}
    with pytest.raises(ValueError):
        B200Config.from_dict({"attention_dp_size": 0})
    with pytest.raises(ValueError):
        B200Config.from_dict({"quantization": "int3"})
    # component / attention DP sizes are accepted (checked against the replicas by the front end)
    assert B200Config.from_dict({"mlp_dp_size": 2, "lm_head_dp_size": 4}).lm_head_dp_size == 4
    # options of the reference that are not implemented are refused, not silently ignored
    for bad in ({"fp8_packed_kv": True}, {"kv_segment_size_buckets": [512]},
                {"decode_context_length_buckets": [1024]}, {"on_device_sampling_config": None}):
        with pytest.raises(NotImplementedError):
            B200Config.from_dict(bad)


def test_arch_config_rope_formats():
    a = ModelArchConfig.from_hf({"rope_parameters": {"rope_theta": 500000.0, "rope_type": "default"},
                                 "hidden_size": 256, "num_attention_heads": 4})
    assert a.rope_theta == 500000.0 and a.rope_scaling is None and a.head_dim == 64
    b = ModelArchConfig.from_hf({"rope_theta": 1e6, "rope_scaling": {"rope_type": "llama3", "factor": 8.0}})
    assert b.rope_theta == 1e6 and b.rope_scaling["factor"] == 8.0
    c = ModelArchConfig.from_hf({"rope_parameters": {"rope_theta": 150000.0, "rope_type": "yarn", "factor": 32.0}})
    assert c.rope_scaling["rope_type"] == "yarn"


def _req(rid, n, max_tokens=4):
    return Request(rid, list(range(1, n + 1)), SamplingParams(temperature=0, max_tokens=max_tokens, ignore_eos=True))


def test_block_manager_alloc_free_and_prefix_cache():
    bm = BlockManager(10, 4, enable_prefix_caching=True)
    r = _req("a", 10)
    assert bm.allocate(r, 10) and len(r.block_ids) == 3 and 0 not in r.block_ids
    r.num_computed_tokens = 10
    bm.commit_full_blocks(r)
    bm.free_request(r)
    assert bm.num_free_blocks == 9
    r2 = _req("b", 10)
    assert bm.match_prefix(r2) == 8  # two full blocks reused
    assert bm.allocate(r2, 10) and len(r2.block_ids) == 3
    big = _req("c", 40)
    assert not bm.allocate(big, 40)  # all-or-nothing
    assert len(big.block_ids) == 0


def test_scheduler_chunked_prefill_and_decode_mix():
    bm = BlockManager(100, 16)
    s = Scheduler(bm, max_num_seqs=4, max_num_batched_tokens=50, max_model_len=512)
    a, b = _req("a", 40), _req("b", 40)
    s.add_request(a)
    s.add_request(b)
    o1 = s.schedule()
    assert [(x.req.request_id, x.num_tokens, x.samples) for x in o1.scheduled] == [("a", 40, True), ("b", 10, False)]
    s.update(o1, [7])
    o2 = s.schedule()
    assert [(x.req.request_id, x.num_tokens) for x in o2.scheduled] == [("a", 1), ("b", 30)]
    s.update(o2, [8, 9])
    assert a.output_token_ids == [7, 8] and b.output_token_ids == [9]


def test_scheduler_no_mixing_mode():
    bm = BlockManager(100, 16)
    s = Scheduler(bm, max_num_seqs=4, max_num_batched_tokens=500, max_model_len=512, mixed_batches=False)
    a, b = _req("a", 20), _req("b", 20)
    s.add_request(a)
    o1 = s.schedule()
    s.update(o1, [1])
    s.add_request(b)
    o2 = s.schedule()
    kinds = {x.num_tokens == 1 for x in o2.scheduled}
    assert len(kinds) == 1  # never prefill and decode together


def test_bucket_for():
    assert bucket_for([128, 256, 512], 1) == 128
    assert bucket_for([128, 256, 512], 300) == 512
    assert bucket_for([128], 600) == 600
    assert bucket_for(None, 7) == 7


def test_parallel_group_math():
    assert ps.tp_groups(8, 4) == [[0, 1, 2, 3], [4, 5, 6, 7]]
    assert ps.dp_groups(8, 4) == [[0, 4], [1, 5], [2, 6], [3, 7]]
    assert ps.ep_groups(8, 8) == [list(range(8))]
    assert ps.ep_tp_groups(8, 4) == [[0, 4], [1, 5], [2, 6], [3, 7]]
    inner, outer = ps.sub_groups(list(range(8)), 2)
    assert inner == [[0, 1], [2, 3], [4, 5], [6, 7]] and outer == [[0, 2, 4, 6], [1, 3, 5, 7]]
    kv, head = ps.dcp_groups(list(range(8)), 2)
    assert kv == [[0, 4], [1, 5], [2, 6], [3, 7]] and head == [[0, 1, 2, 3], [4, 5, 6, 7]]
    with pytest.raises(ValueError):
        ps.ParallelConfig(world_size=8, tensor_parallel_size=3, data_parallel_size=1).validate()


def test_emulated_rank_engine_runs_on_cpu():
    """A single process can run one rank's share of TP=2 (profiling aid) without a process group."""
    from vllm_neuron_b200.engine.llm_engine import EngineArgs, LLMEngine
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.parallel.comm import EmulatedRankComm

    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 64,
           "num_hidden_layers": 1, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 16,
           "intermediate_size": 128, "vocab_size": 256, "max_position_embeddings": 128}
    eng = LLMEngine(EngineArgs(model=cfg, max_num_seqs=2, max_model_len=64, max_num_batched_tokens=64,
                               load_format="dummy", device="cpu", num_gpu_blocks=32, dtype="float32"),
                    tp=EmulatedRankComm(2))
    assert eng.model.Hq == 2 and eng.model.Hkv == 1
    eng.add_request(list(range(10)), SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True))
    done = eng.run_until_done()
    assert len(done) == 1 and len(done[0].output_token_ids) == 3


def test_prompt_logits_matches_hf():
    """The logit-validation hook returns the HF logits of the last prompt position."""
    from tests._tiny import random_prompts, tiny_llama_checkpoint
    from vllm_neuron_b200.entrypoints import LLM

    d, hf = tiny_llama_checkpoint()
    prompts = random_prompts(n=2, length=20)
    llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=32,
              max_num_batched_tokens=128)
    got = llm.engine.prompt_logits(prompts)
    with torch.no_grad():
        ref = torch.stack([hf(torch.tensor([p])).logits[0, -1] for p in prompts])
    assert torch.allclose(got, ref, atol=1e-4, rtol=1e-4)


def test_block_fp8_checkpoint_loads(tmp_path):
    """A Llama checkpoint with block-scaled fp8 weights (+ *_scale_inv) loads and matches the
    dequantized bf16 model's logits."""
    from safetensors.torch import load_file, save_file

    from tests._tiny import random_prompts, tiny_llama_checkpoint
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.utils.checkpoints import dequant_block_fp8, quant_block_fp8
    import json, os, shutil

    d, _ = tiny_llama_checkpoint()
    w = torch.randn(300, 200) * 0.05
    q, s = quant_block_fp8(w)
    assert (dequant_block_fp8(q, s, dtype=torch.float32) - w).abs().max() < 0.05 * w.abs().max()
    out = tmp_path / "fp8"
    shutil.copytree(d, out)
    sd = load_file(str(out / "model.safetensors"))
    deq = {}
    for n, t in list(sd.items()):
        if n.endswith("proj.weight") and t.dim() == 2:
            q, s = quant_block_fp8(t)
            sd[n], sd[n + "_scale_inv"] = q, s
            deq[n] = dequant_block_fp8(q, s, dtype=torch.float32)
    save_file(sd, str(out / "model.safetensors"))
    cfg = json.load(open(out / "config.json"))
    cfg["quantization_config"] = {"quant_method": "fp8", "weight_block_size": [128, 128]}
    json.dump(cfg, open(out / "config.json", "w"))
    ref_dir = tmp_path / "deq"
    shutil.copytree(d, ref_dir)
    sd2 = load_file(str(ref_dir / "model.safetensors"))
    sd2.update(deq)
    save_file(sd2, str(ref_dir / "model.safetensors"))
    kw = dict(device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=32,
              max_num_batched_tokens=128)
    p = random_prompts(n=2, length=10)
    a = LLM(str(out), **kw).engine.prompt_logits(p)
    b = LLM(str(ref_dir), **kw).engine.prompt_logits(p)
    assert torch.allclose(a, b, atol=1e-5)
