"""Decode-path fusions against fp32 oracles.

* SwiGLU finisher of the split-K / stream-K decode GEMM (``ops.linear.gemm_accumulate_silu``):
  the warp that adds the last contribution to a gate/up block pair writes silu(g) * u and zeroes
  the pair's fp32 sums.  Checked for stream-K (more row tiles than SMs) and split-K shapes, batch
  sizes 1..128, and across repeated launches (counters and accumulators must be left zero).
* In-kernel split merge of the decode attention kernel: covered by
  ``test_kernels_gpu.py::test_paged_decode_tma`` (split factors up to 24, repeated launches,
  device split factors); here a decode batch whose launches alternate split factors checks that
  the merge counters are left zero.
"""
import math

import numpy as np
import pytest
import torch

from vllm_neuron_b200 import ops
from vllm_neuron_b200.ops import linear as L

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize("I,K", [(14336, 4096), (1792, 4096), (2048, 1024)])
@pytest.mark.parametrize("M", [1, 7, 64, 128])
def test_gemm_accumulate_silu(cuda_device, I, K, M):
    g = torch.Generator(device=cuda_device).manual_seed(I + M)
    gate = (torch.randn(I, K, device=cuda_device, generator=g) * 0.03).to(torch.bfloat16)
    up = (torch.randn(I, K, device=cuda_device, generator=g) * 0.03).to(torch.bfloat16)
    w = L.interleave_gate_up(gate, up)
    acc = torch.zeros(128, 2 * I, device=cuda_device, dtype=torch.float32)
    ctr = torch.zeros(2 * I // 256, device=cuda_device, dtype=torch.int32)
    out = torch.full((128, I), float("nan"), device=cuda_device, dtype=torch.bfloat16)
    for rep in range(3):
        x = torch.randn(M, K, device=cuda_device, generator=g).to(torch.bfloat16)
        L.gemm_accumulate_silu(x, w, acc[:M], out[:M], ctr)
        torch.cuda.synchronize()
        ref = torch.nn.functional.silu(x.float() @ gate.float().t()) * (x.float() @ up.float().t())
        assert _rel(out[:M], ref) < 1e-2, rep
        assert int(torch.count_nonzero(acc)) == 0 and int(torch.count_nonzero(ctr)) == 0, rep


def test_decode_split_merge_counters(cuda_device):
    Hq, Hkv, D, bs = 32, 8, 128, 16
    ctx = [5, 300, 1000, 64, 2047, 17] * 4
    B = len(ctx)
    g = torch.Generator().manual_seed(0)
    nblk = max((c + bs - 1) // bs for c in ctx)
    nb = B * nblk + 1
    bt = (torch.randperm(nb - 1, generator=g)[: B * nblk] + 1).view(B, nblk).to(torch.int32).to(cuda_device)
    kc = (torch.randn(nb, Hkv, bs, D, generator=g) * 0.5).to(torch.bfloat16).to(cuda_device)
    vc = torch.randn(nb, Hkv, bs, D, generator=g).to(torch.bfloat16).to(cuda_device)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16).to(cuda_device)
    sl = torch.tensor(ctx, dtype=torch.int32, device=cuda_device)
    qs = torch.arange(B + 1, dtype=torch.int32, device=cuda_device)
    w = ops.build_work(np.ones(B), np.array(ctx), Hq // Hkv, Hkv)
    work = torch.from_numpy(w.work).to(cuda_device)
    ref = ops.paged_attention_ref(q, kc, vc, bt, sl, qs, 1 / math.sqrt(D), 0, None)
    for splits in (7, 2, 32, 7, 1, 13):
        out = ops.paged_attention(q, kc, vc, bt, sl, qs, work, True, splits, 1 / math.sqrt(D))
        torch.cuda.synchronize()
        assert _rel(out, ref) < 2e-2, splits
