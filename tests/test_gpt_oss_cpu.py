"""GPT-OSS on CPU (fp32): a tiny GptOssForCausalLM (sliding/full attention alternation, sinks,
YaRN, biased QKV/O, top-k MoE with clamped SwiGLU) must generate the same greedy tokens as the
HF reference, also with the experts split over two emulated expert-parallel shards."""
import tempfile

import torch

from tests._tiny import random_prompts
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM


def _tiny_gpt_oss(seed=0):
    from transformers import GptOssConfig, GptOssForCausalLM

    torch.manual_seed(seed)
    cfg = GptOssConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=16, intermediate_size=96, num_local_experts=4, num_experts_per_tok=2,
                       vocab_size=512, sliding_window=8, max_position_embeddings=512,
                       layer_types=["sliding_attention", "full_attention"], initializer_range=0.05,
                       rope_scaling={"rope_type": "yarn", "factor": 4.0, "beta_fast": 32.0, "beta_slow": 1.0,
                                     "truncate": False, "original_max_position_embeddings": 128})
    hf = GptOssForCausalLM(cfg).float().eval()
    with torch.no_grad():
        for m in hf.modules():
            for n, prm in m.named_parameters(recurse=False):
                if n in ("sinks",) or n.endswith("bias"):
                    prm.normal_(0.0, 0.5)
    d = tempfile.mkdtemp(prefix="tiny_gptoss_")
    hf.save_pretrained(d, safe_serialization=True)
    return d, hf


def _hf_greedy(hf, prompt, n):
    ids = torch.tensor([prompt])
    out = []
    with torch.no_grad():
        for _ in range(n):
            nxt = int(hf(ids).logits[0, -1].argmax())
            out.append(nxt)
            ids = torch.cat([ids, torch.tensor([[nxt]])], 1)
    return out


def test_gpt_oss_generate_matches_hf():
    d, hf = _tiny_gpt_oss()
    prompts = random_prompts(n=3, length=20, vocab=512)
    llm = LLM(d, device="cpu", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64, block_size=16,
              max_num_batched_tokens=64, dtype="float32")
    outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=10, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert o.outputs[0].token_ids == _hf_greedy(hf, p, 10)


def test_mxfp4_roundtrip_matches_transformers_dequant():
    from vllm_neuron_b200.models.gpt_oss import dequant_mxfp4, quant_mxfp4

    w = torch.randn(3, 8, 64) * 0.1
    blocks, scales = quant_mxfp4(w)
    assert blocks.shape == (3, 8, 2, 16) and scales.shape == (3, 8, 2)
    deq = dequant_mxfp4(blocks, scales, torch.float32)
    assert (deq - w).abs().max() <= w.abs().amax() / 4 + 1e-6
    # requantizing the dequantized values is exact
    b2, s2 = quant_mxfp4(deq)
    assert torch.equal(dequant_mxfp4(b2, s2, torch.float32), deq)
    try:
        from transformers.integrations.mxfp4 import convert_moe_packed_tensors
    except Exception:
        return
    ref = convert_moe_packed_tensors(blocks, scales, dtype=torch.float32)
    # transformers returns the transposed [..., K, N] layout of the HF module
    assert torch.equal(ref.transpose(-1, -2).contiguous(), deq) or torch.equal(ref, deq)


def test_mxfp4_kernel_layout_roundtrip():
    """Emulate the MXFP4 kernel's reads of its weight tiles (tile (nb, c): column r's 32 bytes at
    r * 32, lane t's 8 bytes at 8t: byte 2s holds k = 16s + 2t, +1, byte 2s + 1 holds
    k = 16s + 2t + 8, +9; scales at 256 * 32 + 2r)."""
    from vllm_neuron_b200.models.gpt_oss import _FP4_VALUES, dequant_mxfp4, quant_mxfp4
    from vllm_neuron_b200.ops.moe import TILE_COLS, pack_mxfp4

    E, N, K = 2, 300, 128
    w = torch.randn(E, N, K) * 0.3
    blocks, scales = quant_mxfp4(w)
    ref = dequant_mxfp4(blocks, scales, torch.float32)
    wt = pack_mxfp4(blocks, scales)
    assert wt.shape == (E, 2, K // 64, TILE_COLS * 34)
    lut = torch.tensor(_FP4_VALUES)
    got = torch.zeros_like(ref)
    for e in range(E):
        for n in range(N):
            nb, r = divmod(n, TILE_COLS)
            for c in range(K // 64):
                tile = wt[e, nb, c]
                sc = tile[TILE_COLS * 32 + 2 * r:TILE_COLS * 32 + 2 * r + 2].tolist()
                for t in range(4):
                    by = tile[r * 32 + 8 * t:r * 32 + 8 * t + 8].tolist()
                    for s in range(4):
                        f = 2.0 ** (sc[s // 2] - 127)
                        for half, b in enumerate((by[2 * s], by[2 * s + 1])):
                            k = c * 64 + 16 * s + 2 * t + 8 * half
                            got[e, n, k] = lut[b & 15] * f
                            got[e, n, k + 1] = lut[b >> 4] * f
    assert torch.equal(got, ref)
