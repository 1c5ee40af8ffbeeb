"""FP8 (e4m3) KV cache on the GPU: the KV-write kernel's quantization, the persistent TMA
decode kernel and the prefill / chunked-prefill kernel against the fp32 oracle over the same
fp8 cache, and a model served with ``kv_cache_dtype="fp8"``."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_neuron_b200 import ops
from vllm_neuron_b200.ops._ext import ext

K_SCALE, V_SCALE = 0.05, 0.02


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _status(cuda_device):
    torch.manual_seed(0)
    ext().reset_status()
    yield
    torch.cuda.synchronize()
    assert ext().read_status() == 0, "a bounded device wait expired"


def _fp8_batch(device, q_lens, ctx_lens, Hq, Hkv, D, bs=16, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(q_lens)
    seq_lens = [c + q for c, q in zip(ctx_lens, q_lens)]
    max_blocks = max((s + bs - 1) // bs for s in seq_lens)
    nb = B * max_blocks + 3
    bt = (torch.randperm(nb - 1, generator=g)[: B * max_blocks] + 1).view(B, max_blocks).to(torch.int32)
    k = torch.randn(nb, Hkv, bs, D, generator=g) * 0.5
    v = torch.randn(nb, Hkv, bs, D, generator=g)
    kc = ops.attention.quantize_kv_fp8(k, K_SCALE)
    vc = ops.attention.quantize_kv_fp8(v, V_SCALE)
    kc[0].zero_()
    vc[0].zero_()
    q = torch.randn(sum(q_lens), Hq, D, generator=g).to(torch.bfloat16)
    q_start = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    return [t.to(device) for t in (q, kc, vc, bt, sl, q_start)]


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("q_len", [1, 3])
@pytest.mark.parametrize("window,sinks", [(0, False), (100, True)])
def test_fp8_decode_tma(cuda_device, D, q_len, window, sinks):
    Hq, Hkv = {128: (16, 4), 64: (20, 4), 256: (8, 2)}[D]
    ctx = [1, 15, 16, 17, 63, 64, 65, 300, 1000, 2047, 5]
    q_lens = [q_len] * len(ctx)
    q, kc, vc, bt, sl, qs = _fp8_batch(cuda_device, q_lens, ctx, Hq, Hkv, D)
    sink_t = (torch.randn(Hq, device=cuda_device) * 2).float() if sinks else None
    scale = 1 / math.sqrt(D)
    w = ops.build_work(np.array(q_lens), sl.cpu().numpy(), Hq // Hkv, Hkv, head_dim=D)
    assert w.decode
    work = torch.from_numpy(w.work).to(cuda_device)
    ref = ops.paged_attention_ref(q, kc, vc, bt, sl, qs, scale, window, sink_t, K_SCALE, V_SCALE)
    for splits in sorted({1, w.num_splits, 5}):
        for _ in range(2):
            out = ops.paged_attention(q, kc, vc, bt, sl, qs, work, True, splits, scale, window=window,
                                      sinks=sink_t, k_scale=K_SCALE, v_scale=V_SCALE)
            assert _rel_err(out, ref) < 2e-2, splits


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("case", ["prefill", "mixed", "chunked"])
def test_fp8_prefill(cuda_device, D, case):
    Hq, Hkv = {128: (8, 2), 64: (16, 2), 256: (8, 2)}[D]
    q_lens, ctx = {"prefill": ([100, 1, 257, 64], [0, 0, 0, 0]),
                   "mixed": ([1, 1, 90, 1, 33], [400, 20, 0, 1500, 700]),
                   "chunked": ([512, 200], [1024, 300])}[case]
    q, kc, vc, bt, sl, qs = _fp8_batch(cuda_device, q_lens, ctx, Hq, Hkv, D)
    scale = 1 / math.sqrt(D)
    w = ops.build_work(np.array(q_lens), sl.cpu().numpy(), Hq // Hkv, Hkv, head_dim=D)
    work = torch.from_numpy(w.work).to(cuda_device)
    out = ops.paged_attention(q, kc, vc, bt, sl, qs, work, w.decode, w.num_splits, scale,
                              k_scale=K_SCALE, v_scale=V_SCALE)
    ref = ops.paged_attention_ref(q, kc, vc, bt, sl, qs, scale, 0, None, K_SCALE, V_SCALE)
    assert _rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("D", [64, 128, 256])
def test_fp8_kv_write(cuda_device, D):
    T, Hq, Hkv, bs, nb = 20, 8, 2, 16, 8
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=cuda_device, dtype=torch.bfloat16) * 4
    qkv_cpu = qkv.cpu().clone()
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=cuda_device)
    slots = torch.randperm(nb * bs)[:T].to(torch.int32)
    slots[3] = -1
    tab = ops.cos_sin_table(4096, D, 500000.0, device=cuda_device)
    kc = torch.zeros(nb, Hkv, bs, D, device=cuda_device, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(T, Hq * D, device=cuda_device, dtype=torch.bfloat16)
    ops.rope_kv_write(qkv, pos, tab, Hq, Hkv, D, q_out, kc, vc, slots.to(cuda_device),
                      k_scale=K_SCALE * 20, v_scale=V_SCALE * 20)
    kr = torch.zeros(nb, Hkv, bs, D, dtype=torch.float8_e4m3fn)
    vr = torch.zeros_like(kr)
    q_r = torch.empty(T, Hq * D, dtype=torch.bfloat16)
    ops.rope_kv_write_ref(qkv_cpu, pos.cpu(), tab.cpu(), Hq, Hkv, D, q_r, kr, vr, slots, None, None,
                          1e-6, D, True, k_scale=K_SCALE * 20, v_scale=V_SCALE * 20)
    for got, want in ((kc, kr), (vc, vr)):
        g8, w8 = got.cpu().view(torch.uint8), want.view(torch.uint8)
        assert (g8 == w8).float().mean().item() > 0.99  # rounding ties of the fp32 RoPE may differ
        assert _rel_err(got.cpu().float(), want.float()) < 2e-2
    assert _rel_err(q_out.cpu(), q_r) < 1e-2


def test_fp8_kv_llm(cuda_device):
    """A Llama model served with an fp8 cache: prompt logits close to the bf16-cache run, and
    greedy decode through the CUDA-graph path raises no device error."""
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 512,
           "num_hidden_layers": 2, "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 64,
           "intermediate_size": 1024, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
           "max_position_embeddings": 2048}
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (37, 150, 300, 64)]
    logits, toks = {}, {}
    for kv in ("auto", "fp8"):
        llm = LLM(cfg, max_num_seqs=4, max_model_len=1024, num_gpu_blocks=256, load_format="dummy",
                  device="cuda:0", skip_tokenizer_init=True, kv_cache_dtype=kv)
        assert llm.engine.runner.kv_cache.dtype == (torch.float8_e4m3fn if kv == "fp8" else torch.bfloat16)
        logits[kv] = llm.engine.prompt_logits(prompts)
        outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))
        toks[kv] = [o.outputs[0].token_ids for o in outs]
        llm.shutdown()
    assert _rel_err(logits["fp8"], logits["auto"]) < 5e-2
    assert all(len(t) == 16 for t in toks["fp8"])
    # the first sampled token comes from the (nearly identical) prefill logits
    assert sum(a[0] == b[0] for a, b in zip(toks["fp8"], toks["auto"])) >= 3
