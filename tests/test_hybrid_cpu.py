"""Hybrid gated-DeltaNet + gated-attention MoE (Qwen3.5/3.6 family, text) on CPU in fp32 against
HF transformers, including chunked prefill (the recurrent and conv states carry across
chunks) and the op-level oracles of the DeltaNet kernels."""
import tempfile

import torch

from tests._tiny import random_prompts
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM
from vllm_neuron_b200.ops import deltanet as DN


def _tiny_hybrid(seed=0):
    from transformers import Qwen3_5MoeForCausalLM
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig

    torch.manual_seed(seed)
    cfg = Qwen3_5MoeTextConfig(hidden_size=128, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=64, linear_key_head_dim=128, linear_value_head_dim=128,
                               linear_num_key_heads=1, linear_num_value_heads=2, linear_conv_kernel_dim=4,
                               moe_intermediate_size=32, shared_expert_intermediate_size=32, num_experts=8,
                               num_experts_per_tok=2, vocab_size=512, max_position_embeddings=512,
                               initializer_range=0.05, tie_word_embeddings=False,
                               rope_parameters={"rope_type": "default", "rope_theta": 10000.0,
                                                "partial_rotary_factor": 0.25})
    hf = Qwen3_5MoeForCausalLM(cfg).float().eval()
    with torch.no_grad():
        for n, prm in hf.named_parameters():
            if "norm" in n and "linear_attn.norm" not in n:
                prm.normal_(0.0, 0.1)  # exercise the (1 + w) norm convention
    d = tempfile.mkdtemp(prefix="tiny_hybrid_")
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


def test_hybrid_generate_matches_hf():
    d, hf = _tiny_hybrid()
    prompts = random_prompts(n=3, length=30, vocab=512)
    ref = [_hf_greedy(hf, p, 8) for p in prompts]
    for chunk in (256, 16):  # whole-prompt prefill, then chunked prefill across steps
        llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
                  max_num_batched_tokens=chunk)
        outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
        assert [o.outputs[0].token_ids for o in outs] == ref, chunk


def test_conv1d_ref_matches_full_sequence():
    C, K = 6, 4
    x = torch.randn(10, C)
    w = torch.randn(C, K)
    full = torch.nn.functional.silu(torch.nn.functional.conv1d(x.t()[None], w[:, None, :], padding=K - 1,
                                                               groups=C)[0, :, :10].t())
    state = torch.zeros(2, C, K - 1)
    slots = torch.tensor([1], dtype=torch.int32)
    a = DN.causal_conv1d_ref(x[:7], w, torch.tensor([0, 7]), torch.tensor([7]), slots, state)
    b = DN.causal_conv1d_ref(x[7:], w, torch.tensor([0, 3]), torch.tensor([10]), slots, state)
    assert torch.allclose(torch.cat([a, b]), full, atol=1e-5)


def test_chunked_delta_rule_restatement_matches_recurrence():
    """The chunked (WY) form computed by the prefill kernels, restated in torch, equals the
    token-by-token recurrence: outputs and carried state, fresh and continuing sequences."""
    import torch.nn.functional as F

    from vllm_neuron_b200.ops import deltanet as DN

    g = torch.Generator().manual_seed(0)
    Hk, Hv, dk = 2, 4, 128
    q_lens, ctx = [150, 1, 64, 65, 3], [0, 10, 70, 0, 5]
    T = sum(q_lens)
    qkv = torch.randn(T, 2 * Hk * dk + Hv * dk, generator=g)
    a, b = torch.randn(T, Hv, generator=g), torch.randn(T, Hv, generator=g)
    A_log, dt_bias = torch.randn(Hv, generator=g) * 0.5, torch.randn(Hv, generator=g) * 0.3
    qs = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    sl = torch.tensor([c + q for c, q in zip(ctx, q_lens)], dtype=torch.int32)
    slots = torch.tensor([3, 0, 2, 1, 4], dtype=torch.int32)
    st_rec = torch.randn(5, Hv, dk, dk, generator=g) * 0.1
    st_chk = st_rec.clone()
    # recurrence with an identity "norm" (z -> silu^-1 unneeded: compare pre-norm outputs)
    q = qkv[:, :Hk * dk].view(T, Hk, dk).repeat_interleave(Hv // Hk, 1)
    k = qkv[:, Hk * dk:2 * Hk * dk].view(T, Hk, dk).repeat_interleave(Hv // Hk, 1)
    v = qkv[:, 2 * Hk * dk:].view(T, Hv, dk)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    gt = torch.exp(-A_log.exp() * F.softplus(a + dt_bias))
    beta = torch.sigmoid(b)
    o_rec = torch.zeros(T, Hv, dk)
    for bi in range(len(q_lens)):
        t0, t1 = int(qs[bi]), int(qs[bi + 1])
        S = st_rec[slots[bi]].clone() if ctx[bi] > 0 else torch.zeros(Hv, dk, dk)
        for t in range(t0, t1):
            S = S * gt[t][:, None, None]
            d = (v[t] - torch.einsum("hkv,hk->hv", S, k[t])) * beta[t][:, None]
            S = S + k[t][:, :, None] * d[:, None, :]
            o_rec[t] = torch.einsum("hkv,hk->hv", S, q[t])
        st_rec[slots[bi]].copy_(S)
    o_chk = DN.gated_delta_rule_chunked_ref(qkv, a, b, A_log, dt_bias, qs, sl, slots, st_chk, Hk, Hv)
    assert ((o_chk - o_rec).norm() / o_rec.norm()).item() < 1e-5
    assert ((st_chk - st_rec).norm() / st_rec.norm()).item() < 1e-5
