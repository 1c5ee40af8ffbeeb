"""Numerics of every sm_100a kernel against a plain fp32 PyTorch reference of the same op."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_neuron_b200 import ops
from vllm_neuron_b200.ops import linear as L
from vllm_neuron_b200.ops._ext import ext


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _seed_and_status(cuda_device):
    torch.manual_seed(0)
    ext().reset_status()
    yield
    torch.cuda.synchronize()
    assert ext().read_status() == 0, "a bounded device wait expired"


# ----------------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (1000, 384, 4096),
                                   (4096, 6144, 4096), (300, 1000, 200), (129, 2048, 136)])
@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_wide(cuda_device, M, N, K, bn):
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    out = L.gemm_out(x, w, bn=bn)
    ref = x.float() @ w.float().t()
    assert _rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("M", [1, 7, 16, 33, 64, 100, 128])
@pytest.mark.parametrize("N,K", [(768, 4096), (4096, 14336), (6144, 4096), (1000, 72)])
def test_gemm_skinny_and_splitk(cuda_device, M, N, K):
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    ref = x.float() @ w.float().t()
    out = L.gemm_skinny_bf16(x, w)
    assert _rel_err(out, ref) < 1e-2
    acc = torch.zeros(M, N, device=cuda_device, dtype=torch.float32)
    L.gemm_accumulate(x, w, acc)  # stream-K
    assert _rel_err(acc, ref) < 1e-3
    acc.zero_()
    L.gemm_accumulate(x, w, acc, splits=3)  # fixed split-K
    assert _rel_err(acc, ref) < 1e-3


def test_gemm_accumulate_wide_splitk(cuda_device):
    M, N, K = 512, 768, 8192
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    acc = torch.zeros(M, N, device=cuda_device, dtype=torch.float32)
    L.gemm_accumulate(x, w, acc, splits=4)
    assert _rel_err(acc, x.float() @ w.float().t()) < 1e-3
    acc.zero_()
    L.gemm_accumulate(x, w, acc)  # stream-K over wide tiles
    assert _rel_err(acc, x.float() @ w.float().t()) < 1e-3


@pytest.mark.parametrize("M,I,K", [(256, 512, 1024), (1000, 1792, 4096), (130, 256, 64)])
def test_gemm_silu_epilogue(cuda_device, M, I, K):
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    g = torch.randn(I, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    u = torch.randn(I, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    w = L.interleave_gate_up(g, u)
    out = L.gemm_silu(x, w)
    ref = torch.nn.functional.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())
    assert _rel_err(out, ref) < 1e-2


# ------------------------------------------------------------------------------ attention
def _make_batch(device, q_lens, ctx_lens, Hq, Hkv, D, bs=16, num_blocks=None, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(q_lens)
    seq_lens = [c + q for c, q in zip(ctx_lens, q_lens)]
    max_blocks = max((s + bs - 1) // bs for s in seq_lens)
    nb = num_blocks or (B * max_blocks + 3)
    perm = torch.randperm(nb - 1, generator=g)[: B * max_blocks] + 1
    bt = perm.view(B, max_blocks).to(torch.int32)
    k_cache = (torch.randn(nb, Hkv, bs, D, generator=g) * 0.5).to(torch.bfloat16).to(device)
    v_cache = torch.randn(nb, Hkv, bs, D, generator=g).to(torch.bfloat16).to(device)
    T = sum(q_lens)
    q = torch.randn(T, Hq, D, generator=g).to(torch.bfloat16).to(device)
    q_start = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32)
    return q, k_cache, v_cache, bt.to(device), torch.tensor(seq_lens, dtype=torch.int32).to(device), q_start.to(device)


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("bs", [16, 32])
@pytest.mark.parametrize("q_len", [1, 3])
@pytest.mark.parametrize("window,sinks", [(0, False), (100, True)])
def test_paged_decode_tma(cuda_device, D, bs, q_len, window, sinks):
    """Decode batches run the persistent TMA kernel (contiguous caches, block_size % 16 == 0);
    several split factors, including splits that are empty for short sequences."""
    Hq, Hkv = {128: (16, 4), 64: (20, 4), 256: (8, 2)}[D]
    ctx = [1, 15, 16, 17, 63, 64, 65, 300, 1000, 2047, 5]
    q_lens = [q_len] * len(ctx)
    q, kc, vc, bt, sl, qs = _make_batch(cuda_device, q_lens, ctx, Hq, Hkv, D, bs=bs)
    sink_t = (torch.randn(Hq, device=cuda_device) * 2).float() if sinks else None
    scale = 1 / math.sqrt(D)
    w = ops.build_work(np.array(q_lens), sl.cpu().numpy(), Hq // Hkv, Hkv)
    assert w.decode
    work = torch.from_numpy(w.work).to(cuda_device)
    ref = ops.paged_attention_ref(q, kc, vc, bt, sl, qs, scale, window, sink_t)
    for splits in sorted({1, w.num_splits, 5, 24}):
        for _ in range(2):  # the unit counter must be reset between launches
            out = ops.paged_attention(q, kc, vc, bt, sl, qs, work, True, splits, scale,
                                      window=window, sinks=sink_t)
            assert _rel_err(out, ref) < 2e-2, splits
    # a device-side split factor below the launch's (CUDA-graph decode): 1 and 3 of 24
    for dev_splits in (1, 3):
        sd = torch.tensor([dev_splits], dtype=torch.int32, device=cuda_device)
        out = ops.paged_attention(q, kc, vc, bt, sl, qs, work, True, 24, scale, window=window,
                                  sinks=sink_t, splits_dev=sd)
        assert _rel_err(out, ref) < 2e-2, dev_splits


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("case", ["prefill", "decode", "mixed", "chunked"])
@pytest.mark.parametrize("window,sinks", [(0, False), (128, True), (0, True)])
def test_paged_attention(cuda_device, D, case, window, sinks):
    Hq, Hkv = {128: (8, 2), 64: (16, 2), 256: (8, 2)}[D]
    if case == "prefill":
        q_lens, ctx = [100, 1, 257, 64], [0, 0, 0, 0]
    elif case == "decode":
        q_lens, ctx = [1] * 9, [5, 17, 300, 1000, 64, 65, 127, 2000, 3]
    elif case == "mixed":
        q_lens, ctx = [1, 1, 90, 1, 33], [400, 20, 0, 1500, 700]
    else:
        q_lens, ctx = [512, 200], [1024, 300]
    q, kc, vc, bt, sl, qs = _make_batch(cuda_device, q_lens, ctx, Hq, Hkv, D)
    sink_t = (torch.randn(Hq, device=cuda_device) * 2).float() if sinks else None
    scale = 1 / math.sqrt(D)
    w = ops.build_work(np.array(q_lens), sl.cpu().numpy(), Hq // Hkv, Hkv)
    work = torch.from_numpy(w.work).to(cuda_device)
    out = ops.paged_attention(q, kc, vc, bt, sl, qs, work, w.decode, w.num_splits, scale,
                              window=window, sinks=sink_t)
    ref = ops.paged_attention_ref(q, kc, vc, bt, sl, qs, scale, window, sink_t)
    assert _rel_err(out, ref) < 2e-2


def test_paged_attention_forced_splits(cuda_device):
    q_lens, ctx = [1, 1, 1], [3000, 50, 777]
    q, kc, vc, bt, sl, qs = _make_batch(cuda_device, q_lens, ctx, 32, 8, 128)
    w = ops.build_work(np.array(q_lens), sl.cpu().numpy(), 4, 8)
    work = torch.from_numpy(w.work).to(cuda_device)
    ref = ops.paged_attention_ref(q, kc, vc, bt, sl, qs, 0.088)
    for splits in (1, 2, 8):
        out = ops.paged_attention(q, kc, vc, bt, sl, qs, work, True, splits, 0.088)
        assert _rel_err(out, ref) < 2e-2


# --------------------------------------------------------------------- norm / rope / misc
@pytest.mark.parametrize("H", [256, 2880, 4096, 8192])
@pytest.mark.parametrize("f32_in", [False, True])
def test_add_rmsnorm(cuda_device, H, f32_in):
    T = 37
    x = torch.randn(T, H, device=cuda_device, dtype=torch.float32 if f32_in else torch.bfloat16)
    res = torch.randn(T, H, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(H, device=cuda_device, dtype=torch.bfloat16)
    res_ref = (res.float() + x.float()).to(torch.bfloat16)
    ref = ops.rmsnorm_ref(res_ref, w, 1e-5)
    out = ops.add_rmsnorm(x, res, w, 1e-5, clear_x=True)
    assert torch.equal(res, res_ref)
    assert _rel_err(out, ref) < 1e-2
    if f32_in:
        assert torch.count_nonzero(x) == 0
    out2 = ops.rmsnorm(res, w, 1e-5)
    assert _rel_err(out2, ref) < 1e-2


@pytest.mark.parametrize("D,neox,qknorm,f32_in,rot,T,Hq,Hkv", [
    (128, True, False, False, None, 20, 8, 2), (128, True, True, True, None, 20, 8, 2),
    (64, True, False, True, None, 20, 8, 2), (128, False, False, False, None, 20, 8, 2),
    (256, True, True, False, None, 20, 8, 2),
    (128, True, False, False, None, 300, 32, 8),   # two head groups per token (vector kernel)
    (128, False, False, True, 64, 40, 8, 2),       # interleaved, partial rotary (vector kernel)
    (128, True, False, False, 64, 40, 8, 2),       # neox, partial rotary (per-head kernel)
])
def test_rope_kv_write(cuda_device, D, neox, qknorm, f32_in, rot, T, Hq, Hkv):
    bs, nb = 16, (T + 15) // 16 + 4
    rot = rot or D
    dt = torch.float32 if f32_in else torch.bfloat16
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=cuda_device, dtype=dt)
    qkv_cpu = qkv.detach().cpu().clone()
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=cuda_device)
    slots = torch.randperm(nb * bs)[:T].to(torch.int32)
    slots[3] = -1
    slots = slots.to(cuda_device)
    tab = ops.cos_sin_table(4096, rot, 500000.0, device=cuda_device)
    qn = torch.randn(D, device=cuda_device, dtype=torch.bfloat16) if qknorm else None
    kn = torch.randn(D, device=cuda_device, dtype=torch.bfloat16) if qknorm else None
    kc = torch.zeros(nb, Hkv, bs, D, device=cuda_device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(T, Hq * D, device=cuda_device, dtype=torch.bfloat16)
    ops.rope_kv_write(qkv, pos, tab, Hq, Hkv, D, q_out, kc, vc, slots, qn, kn, 1e-6, neox=neox,
                      clear_input=True, rot_dim=rot)
    kc_r = torch.zeros(nb, Hkv, bs, D, dtype=torch.bfloat16)
    vc_r = torch.zeros_like(kc_r)
    q_r = torch.empty(T, Hq * D, dtype=torch.bfloat16)
    ops.rope_kv_write_ref(qkv_cpu, pos.cpu(), tab.cpu(), Hq, Hkv, D, q_r, kc_r, vc_r, slots.cpu(),
                          qn.cpu() if qknorm else None, kn.cpu() if qknorm else None, 1e-6, rot, neox)
    assert _rel_err(q_out.cpu(), q_r) < 1e-2
    assert _rel_err(kc.cpu(), kc_r) < 1e-2
    assert _rel_err(vc.cpu(), vc_r) < 1e-2
    if f32_in:
        assert torch.count_nonzero(qkv) == 0


@pytest.mark.parametrize("blk,act,f32_in", [(0, 0, False), (128, 0, True), (0, 1, False), (128, 1, True)])
def test_silu_mul(cuda_device, blk, act, f32_in):
    T, I = 19, 1792
    x = torch.randn(T, 2 * I, device=cuda_device, dtype=torch.float32 if f32_in else torch.bfloat16) * 3
    xc = x.cpu().clone()
    out = ops.silu_mul(x, blk=blk, clear_input=True, act=act)
    ref = ops.silu_mul(xc, blk=blk, act=act)
    assert _rel_err(out.cpu(), ref) < 1e-2


def test_embedding(cuda_device):
    V, H = 1000, 512
    table = torch.randn(V, H, device=cuda_device, dtype=torch.bfloat16)
    ids = torch.randint(0, 2 * V, (33,), dtype=torch.int32, device=cuda_device)
    out = ops.embedding(ids, table, vocab_start=500, vocab_end=1500)
    ref = ops.embedding(ids.cpu(), table.cpu(), vocab_start=500, vocab_end=1500)
    assert torch.equal(out.cpu(), ref)


def test_sampling_greedy_and_argmax(cuda_device):
    B, V = 11, 128256
    logits = torch.randn(B, V, device=cuda_device, dtype=torch.bfloat16)
    z = torch.zeros(B, device=cuda_device)
    tk = torch.zeros(B, dtype=torch.int32, device=cuda_device)
    tp = torch.ones(B, device=cuda_device)
    seeds = torch.arange(B, dtype=torch.int64, device=cuda_device)
    offs = torch.zeros(B, dtype=torch.int32, device=cuda_device)
    tok = ops.sample(logits, z, tk, tp, seeds, offs)
    ref = logits.float().argmax(-1).to(torch.int32)
    assert torch.equal(tok, ref)
    assert torch.equal(ops.argmax(logits), ref)


def test_sampling_topk_topp_support(cuda_device):
    """Sampled tokens always lie inside the top-k / top-p set and follow its distribution."""
    B, V = 4, 5000
    logits = torch.randn(B, V, device=cuda_device) * 3
    temp = torch.tensor([1.0, 0.7, 1.3, 1.0], device=cuda_device)
    tk = torch.tensor([10, 0, 50, 5], dtype=torch.int32, device=cuda_device)
    tp = torch.tensor([1.0, 0.5, 0.9, 0.8], device=cuda_device)
    seeds = torch.arange(B, dtype=torch.int64, device=cuda_device)
    counts = torch.zeros(B, V)
    n = 400
    for step in range(n):
        offs = torch.full((B,), step, dtype=torch.int32, device=cuda_device)
        tok = ops.sample(logits, temp, tk, tp, seeds, offs).cpu()
        counts[torch.arange(B), tok.long()] += 1
    from vllm_neuron_b200.ops.sampling import filter_mask_ref
    for b in range(B):
        x = logits[b].cpu() / temp[b].cpu()
        keep = filter_mask_ref(x, int(tk[b]), float(tp[b]), 0.0)
        assert counts[b][~keep].sum() == 0
        p = torch.softmax(x.masked_fill(~keep, float("-inf")), -1)
        top = torch.argmax(p)
        assert abs(counts[b, top] / n - p[top]) < 0.1
    # Same seed and offset reproduce the same tokens.
    offs = torch.full((B,), 7, dtype=torch.int32, device=cuda_device)
    assert torch.equal(ops.sample(logits, temp, tk, tp, seeds, offs),
                       ops.sample(logits, temp, tk, tp, seeds, offs))


def test_device_resident_tokens(cuda_device):
    """Negative ids read the request slot's last sampled token; the sampler writes slots."""
    V, H = 1000, 256
    table = torch.randn(V, H, device=cuda_device, dtype=torch.bfloat16)
    last = torch.zeros(8, dtype=torch.int32, device=cuda_device)
    logits = torch.randn(3, V, device=cuda_device)
    z = torch.zeros(3, device=cuda_device)
    tk = torch.zeros(3, dtype=torch.int32, device=cuda_device)
    tp = torch.ones(3, device=cuda_device)
    sd = torch.zeros(3, dtype=torch.int64, device=cuda_device)
    slots = torch.tensor([5, 2, 7], dtype=torch.int32, device=cuda_device)
    tok = ops.sample(logits, z, tk, tp, sd, tk, row_slots=slots, last_tok=last)
    assert torch.equal(last[slots.long()], tok)
    ids = torch.tensor([-(5 + 1), 17, -(7 + 1)], dtype=torch.int32, device=cuda_device)
    out = ops.embedding(ids, table, last_tok=last)
    assert torch.equal(out[0], table[tok[0]]) and torch.equal(out[1], table[17]) and torch.equal(out[2], table[tok[2]])


def test_apply_token_bitmask(cuda_device):
    from vllm_neuron_b200.ops.sampling import apply_token_bitmask

    V = 1000
    logits = torch.randn(5, V, device=cuda_device).to(torch.bfloat16)
    mask = torch.randint(-2**31, 2**31 - 1, (5, (V + 31) // 32), dtype=torch.int32)
    ref = logits.cpu().float().clone()
    apply_token_bitmask(ref, mask)
    apply_token_bitmask(logits, mask.to(cuda_device))
    assert torch.equal(torch.isinf(logits.cpu().float()), torch.isinf(ref))


def test_bounded_peer_wait_expires_and_context_survives(cuda_device):
    """A fused-collective flag wait whose flag nothing sets gives up after its budget, records
    the peer-flag timeout code in the status word and returns; the context keeps working."""
    import time

    from vllm_neuron_b200.ops._ext import ext

    e = ext()
    e.reset_status()
    flag = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    result = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    t0 = time.perf_counter()
    e.flag_wait_probe(flag, 1, 100.0, result)  # 100 ms budget, nobody sets the flag
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(result.item()) == 0
    assert e.read_status() == 5  # kTimeoutPeerFlag
    assert dt < 5.0
    e.reset_status()
    flag.fill_(1)
    e.flag_wait_probe(flag, 1, 100.0, result)
    torch.cuda.synchronize()
    assert int(result.item()) == 1 and e.read_status() == 0
    # the context is intact: an ordinary kernel still runs and is correct
    x = torch.randn(64, 256, device=cuda_device, dtype=torch.bfloat16)
    w = torch.ones(256, device=cuda_device, dtype=torch.bfloat16)
    y = ops.rmsnorm(x, w, 1e-5)
    ref = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5))
    assert torch.allclose(y.float(), ref, atol=3e-2, rtol=3e-2)


def test_rope_query_position_scale(cuda_device):
    """Long-context query temperature 1 + beta * log(1 + floor(pos / period)) and the fused
    qkv bias in the rope kernel."""
    T, Hq, Hkv, D, bs, nb = 24, 4, 2, 128, 16, 4
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=cuda_device, dtype=torch.bfloat16)
    qkv_cpu = qkv.cpu().clone()
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=cuda_device)
    tab = ops.cos_sin_table(4096, D, 1e6, device=cuda_device)
    q_out = torch.empty(T, Hq * D, device=cuda_device, dtype=torch.bfloat16)
    bias = torch.randn((Hq + 2 * Hkv) * D, device=cuda_device) * 0.5  # fused qkv bias
    ops.rope_kv_write(qkv, pos, tab, Hq, Hkv, D, q_out, q_pos_scale=(0.1, 256.0), qkv_bias=bias)
    q_r = torch.empty(T, Hq * D, dtype=torch.bfloat16)
    ops.rope_kv_write_ref(qkv_cpu.float() + bias.cpu(), pos.cpu(), tab.cpu(), Hq, Hkv, D, q_r, None, None,
                          None, None, None, 1e-6, D, True, (0.1, 256.0))
    assert _rel_err(q_out.cpu(), q_r) < 1e-2
