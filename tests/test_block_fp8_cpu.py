"""Block-scaled FP8 (128 x 128) weights on the CPU: quantization round trip, the GEMM oracles
and a tiny Llama served through ``LLM.generate`` with ``quantization="fp8_block"``."""
import torch

from vllm_neuron_b200.ops import linear as L
from vllm_neuron_b200.utils.checkpoints import dequant_block_fp8, quant_block_fp8


def test_quantize_round_trip_matches_checkpoint_layout():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(300, 520, generator=g) * 0.03
    bw = L.BlockFP8Weight.from_weight(w)
    assert bw.q.shape == (300, 520) and bw.scales.shape == (3, 5)
    # same bytes and scales as the checkpoint-side quantizer
    q, s = quant_block_fp8(w)
    assert torch.equal(bw.q.view(torch.uint8), q.view(torch.uint8))
    assert torch.allclose(bw.scales, s)
    d = bw.dequant()
    assert torch.allclose(d, dequant_block_fp8(q, s, dtype=torch.float32))
    assert float((d - w).norm() / w.norm()) < 0.05
    # an aligned block-FP8 weight re-quantizes to the same bytes (checkpoints load exactly)
    q2 = L.BlockFP8Weight.from_weight(bw.dequant_bf16_ref())
    assert torch.equal(q2.q.view(torch.uint8), bw.q.view(torch.uint8))


def test_cpu_gemm_paths_use_bf16_operands():
    g = torch.Generator().manual_seed(1)
    w = L.BlockFP8Weight.from_weight(torch.randn(256, 384, generator=g) * 0.05)
    x = torch.randn(7, 384, generator=g).to(torch.bfloat16)
    ref = x.float() @ w.dequant_bf16_ref().float().t()
    out = L.gemm_out(x, w, out=torch.empty(7, 256, dtype=torch.bfloat16))
    assert torch.allclose(out.float(), ref, rtol=1e-2, atol=1e-2)
    acc = torch.zeros(7, 256)
    L.gemm_accumulate(x, w, acc)
    assert torch.allclose(acc, ref, rtol=1e-5, atol=1e-5)


def test_tiny_llama_fp8_block_generate():
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 256,
           "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
           "intermediate_size": 512, "vocab_size": 1000, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
           "max_position_embeddings": 256}
    kw = dict(max_num_seqs=4, max_model_len=128, max_num_batched_tokens=128, num_gpu_blocks=64,
              load_format="dummy", device="cpu", skip_tokenizer_init=True, dtype="float32")
    ref = LLM(cfg, **kw)
    q = LLM(cfg, additional_config={"b200_config": {"quantization": "fp8_block"}}, **kw)
    assert all(isinstance(ly.gate_up, L.BlockFP8Weight) for ly in q.engine.model.layers)
    prompts = [[1, 2, 3, 4, 5, 6, 7, 8], [9, 10, 11, 12]]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    a = [o.outputs[0].token_ids for o in ref.generate(prompts, sp)]
    b = [o.outputs[0].token_ids for o in q.generate(prompts, sp)]
    assert all(len(x) == 6 for x in b)
    assert a[0][0] == b[0][0] and a[1][0] == b[1][0]


def test_tiny_hybrid_fp8_block_runs():
    """The hybrid (DeltaNet + gated attention + MoE) with block-FP8 projections gives the logits
    of the same model whose weights are the dequantized bf16 operands (the plumbing is exact;
    the quantization error itself is the checkpoint's)."""
    from tests.test_hybrid_cpu import _tiny_hybrid
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    d, _ = _tiny_hybrid()
    kw = dict(device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=64)
    prompts = [[3, 5, 7, 11, 13, 17, 19, 23] * 3, [2, 4, 6, 8, 10]]
    q = LLM(d, additional_config={"b200_config": {"quantization": "fp8_block"}}, **kw)
    m = q.engine.model
    assert any(isinstance(getattr(ly, "w_in", None), L.BlockFP8Weight) for ly in m.layers)
    assert any(isinstance(getattr(ly, "qkvg", None), L.BlockFP8Weight) for ly in m.layers)
    ref_llm = LLM(d, **kw)
    with torch.no_grad():
        for lq, lr in zip(m.layers, ref_llm.engine.model.layers):
            for name in m.BLOCK_FP8_PARAMS:
                w = getattr(lq, name, None)
                if isinstance(w, L.BlockFP8Weight):
                    getattr(lr, name).copy_(w.dequant_bf16_ref().float())
    got = q.engine.prompt_logits(prompts)
    ref = ref_llm.engine.prompt_logits(prompts)
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-4)
    outs = q.generate(prompts, SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
    assert all(len(o.outputs[0].token_ids) == 5 for o in outs)
