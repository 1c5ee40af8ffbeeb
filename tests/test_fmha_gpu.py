"""tcgen05 prefill attention (csrc/attn/fmha_sm100.cu) against the fp32 oracle.

Head dim 128 with a bf16 cache runs prefill and chunked-prefill steps on the tensor-core kernel
(256 packed query rows per work item as two 128-row Q tiles, 128-token KV tiles, S / P / O in
TMEM, V read MN-major).  Cases: GQA groups 1, 4, 8 and 16, several sequences with cached context
(chunked prefill), sliding windows (narrower than a tile and spanning several), learned sinks,
block sizes 16, 32, 64 and 128, items whose second Q tile is empty, queries past a KV tile
boundary, a single-token prefill among long ones and a 4k-token sequence.  Also checks the bounds
guard: a block table entry beyond the cache is read as the null block and reported in the device
status word.
"""
import math

import numpy as np
import pytest
import torch

from vllm_neuron_b200 import ops
from vllm_neuron_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def _case(dev, q_lens, ctx_lens, Hq, Hkv, bs=16, seed=0, window=0, sinks=False, bad_block=False):
    D = 128
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(q_lens)
    seq_lens = [c + q for c, q in zip(ctx_lens, q_lens)]
    max_blocks = max((s + bs - 1) // bs for s in seq_lens)
    nb = B * max_blocks + 2
    bt = (torch.randperm(nb - 1, generator=g)[: B * max_blocks] + 1).view(B, max_blocks).to(torch.int32)
    kc = (torch.randn(nb, Hkv, bs, D, generator=g) * 0.7).to(torch.bfloat16)
    vc = torch.randn(nb, Hkv, bs, D, generator=g).to(torch.bfloat16)
    q = torch.randn(sum(q_lens), Hq, D, generator=g).to(torch.bfloat16)
    qs = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    sk = (torch.randn(Hq, generator=g) * 2).float() if sinks else None
    scale = 1 / math.sqrt(D)
    rows = ops.attention.prefill_rows(D, torch.bfloat16)
    assert rows == 256
    w = ops.build_work(np.array(q_lens), np.array(seq_lens), Hq // Hkv, Hkv, head_dim=D, prefill_rows=rows)
    assert not w.decode
    ref = ops.paged_attention_ref(q, kc, vc, bt, sl, qs, scale, window, sk)
    if bad_block:  # an entry past the cache (inside the allocation, so nothing unsafe is read)
        kc_big = torch.cat([kc, kc[:1]]).contiguous()
        vc_big = torch.cat([vc, vc[:1]]).contiguous()
        bt2 = bt.clone()
        bt2[0, 0] = nb  # names the extra block, which is beyond the cache the kernel is told
        out = ops.paged_attention(q.to(dev), kc_big[:nb].to(dev), vc_big[:nb].to(dev), bt2.to(dev), sl.to(dev),
                                  qs.to(dev), torch.from_numpy(w.work).to(dev), False, 1, scale,
                                  window=window, sinks=sk.to(dev) if sk is not None else None,
                                  prefill_rows=rows)
        return out, ref
    out = ops.paged_attention(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), sl.to(dev), qs.to(dev),
                              torch.from_numpy(w.work).to(dev), False, 1, scale, window=window,
                              sinks=sk.to(dev) if sk is not None else None, prefill_rows=rows)
    return out, ref


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize("q_lens,ctx,Hq,Hkv,bs,window,sinks", [
    ([200], [0], 32, 8, 16, 0, False),
    ([77, 300, 1], [0, 0, 0], 32, 8, 16, 0, False),
    ([64, 129, 33], [100, 1000, 7], 64, 8, 16, 0, False),       # chunked prefill, G = 8
    ([250, 40], [0, 500], 16, 4, 32, 0, False),                  # block size 32
    ([300, 90], [0, 200], 64, 8, 16, 128, True),                 # sliding window + sinks
    ([1000], [2000], 32, 8, 16, 0, True),
    ([20, 31], [0, 5], 32, 8, 16, 0, False),                     # second Q tile empty
    ([513, 130], [0, 64], 8, 8, 64, 0, False),                   # G = 1, block size 64
    ([96, 300], [10, 0], 64, 4, 128, 0, False),                  # G = 16, block size 128
    ([700], [300], 32, 8, 16, 100, False),                       # window narrower than a KV tile
    ([4096], [0], 32, 8, 16, 0, False),
])
def test_fmha_prefill_matches_oracle(cuda_device, q_lens, ctx, Hq, Hkv, bs, window, sinks):
    out, ref = _case(cuda_device, q_lens, ctx, Hq, Hkv, bs=bs, window=window, sinks=sinks)
    torch.cuda.synchronize()
    assert int(ext().read_status()) == 0
    assert _rel(out, ref) < 2e-2


def test_fmha_block_guard_reports_and_skips(cuda_device):
    ext().reset_status()
    out, _ = _case(cuda_device, [40], [0], 32, 8, bad_block=True)
    torch.cuda.synchronize()
    assert int(ext().read_status()) == 6  # kBadIndex
    assert torch.isfinite(out.float()).all()
    ext().reset_status()
