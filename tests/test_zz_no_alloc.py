"""The allocation-free paged-attention entry point, called through its exported C symbol.

``b200_paged_attention_noalloc`` (csrc/attn/paged_attention_noalloc.cu) is for callers that
cannot allocate device memory while they attend: a host runtime with its own fixed memory
pool, a plain C/C++ host without torch, or a step where a cudaMalloc could stall or fail.
It keeps the split-KV partials in a fixed 16 MiB array in the library instead of asking an
allocator.  This test loads the extension's shared object with ctypes, calls the symbol
twice in a row on different batches (the second call must not see the first call's
leftovers in the shared array) and compares each result with the allocating Python op on
the same inputs, and checks that an oversized call is refused with a message.

The file name sorts last so a run that stops at the first failure has run every other test.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_neuron_b200 import ops
from vllm_neuron_b200.ops._ext import ext, so_path

SCRATCH_BYTES = 16 << 20
ERR_TOO_LARGE = 2


def _lib():
    ext()  # loads the extension (and torch's libraries it links against)
    lib = ctypes.CDLL(so_path())
    fn = lib.b200_paged_attention_noalloc
    fn.restype = ctypes.c_int
    ll, i, p, f = ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p, ctypes.c_float
    fn.argtypes = [p, ll, p, p, ll, p, i, p, p, p, i, p, ll, p, i, i, i, i, i, i, f, i, i, p,
                   ctypes.c_char_p, ctypes.c_size_t]
    return fn


def _batch(device, ctx_lens, Hq, Hkv, D, bs=16, seed=0, q_lens=None):
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(ctx_lens)
    q_lens = list(q_lens) if q_lens is not None else [1] * B
    seq_lens = [c + n for c, n in zip(ctx_lens, q_lens)]
    max_blocks = max((s + bs - 1) // bs for s in seq_lens)
    nb = B * max_blocks + 3
    bt = (torch.randperm(nb - 1, generator=g)[: B * max_blocks] + 1).view(B, max_blocks)
    kc = (torch.randn(nb, Hkv, bs, D, generator=g) * 0.5).to(torch.bfloat16).to(device)
    vc = torch.randn(nb, Hkv, bs, D, generator=g).to(torch.bfloat16).to(device)
    q = torch.randn(sum(q_lens), Hq, D, generator=g).to(torch.bfloat16).to(device)
    qs = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32, device=device)
    sl = torch.tensor(seq_lens, dtype=torch.int32, device=device)
    return q, kc, vc, bt.to(torch.int32).to(device), sl, qs, np.array(q_lens)


def _call(fn, q, kc, vc, bt, sl, qs, work, decode, splits, scale, window=0, sinks=None,
          out=None):
    err = ctypes.create_string_buffer(256)
    if out is None:
        out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.stride(0), bt.data_ptr(),
            bt.stride(0), sl.data_ptr(), qs.data_ptr(), work.data_ptr(), work.shape[0],
            out.data_ptr(), out.stride(0), sinks.data_ptr() if sinks is not None else None,
            q.shape[0], q.shape[1], kc.shape[1], q.shape[2], kc.shape[2], window, scale,
            int(decode), splits, stream, err, len(err))
    return rc, err.value.decode(), out


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def test_noalloc_matches_allocating_op_twice(cuda_device):
    fn = _lib()
    Hq, Hkv, D = 32, 8, 128
    cases = [
        # (context lengths, window, sinks, seed)
        ([300, 1000, 2000, 17, 64, 129, 777, 1500], 0, False, 1),
        ([40, 900, 3000, 5, 2047, 64], 128, True, 2),
    ]
    for ctx, window, use_sinks, seed in cases:
        q, kc, vc, bt, sl, qs, q_lens = _batch(cuda_device, ctx, Hq, Hkv, D, seed=seed)
        sinks = (torch.randn(Hq, device=cuda_device) * 2).float() if use_sinks else None
        w = ops.build_work(q_lens, sl.cpu().numpy(), Hq // Hkv, Hkv)
        assert w.decode
        splits = max(4, w.num_splits)  # the split-KV path is the one that needs scratch
        work = torch.from_numpy(w.work).to(cuda_device)
        scale = 1 / math.sqrt(D)
        ref = ops.paged_attention(q, kc, vc, bt, sl, qs, work, True, splits, scale,
                                  window=window, sinks=sinks)
        rc, msg, out = _call(fn, q, kc, vc, bt, sl, qs, work, True, splits, scale, window, sinks)
        torch.cuda.synchronize()
        assert rc == 0, msg
        assert _rel_err(out, ref) < 2e-2
        oracle = ops.paged_attention_ref(q, kc, vc, bt, sl, qs, scale, window, sinks)
        assert _rel_err(out, oracle) < 2e-2


def test_noalloc_rejects_oversized_scratch(cuda_device):
    fn = _lib()
    Hq, Hkv, D = 32, 8, 128
    q, kc, vc, bt, sl, qs, q_lens = _batch(cuda_device, [100] * 64, Hq, Hkv, D)
    w = ops.build_work(q_lens, sl.cpu().numpy(), Hq // Hkv, Hkv)
    work = torch.from_numpy(w.work).to(cuda_device)
    splits = 64  # 64 * 64 tokens * 32 heads * 129 floats * 4 B > 16 MiB
    assert 4 * splits * 64 * Hq * (D + 1) > SCRATCH_BYTES
    rc, msg, _ = _call(fn, q, kc, vc, bt, sl, qs, work, True, splits, 1 / math.sqrt(D))
    assert rc == ERR_TOO_LARGE
    assert "scratch" in msg


def _check(fn, device, ctx, Hq, Hkv, D, splits=None, q_lens=None, seed=0):
    q, kc, vc, bt, sl, qs, ql = _batch(device, ctx, Hq, Hkv, D, seed=seed, q_lens=q_lens)
    w = ops.build_work(ql, sl.cpu().numpy(), Hq // Hkv, Hkv, head_dim=D)
    splits = splits if splits is not None else w.num_splits
    work = torch.from_numpy(w.work).to(device)
    scale = 1 / math.sqrt(D)
    ref = ops.paged_attention(q, kc, vc, bt, sl, qs, work, w.decode, splits, scale)
    rc, msg, out = _call(fn, q, kc, vc, bt, sl, qs, work, w.decode, splits, scale)
    torch.cuda.synchronize()
    assert rc == 0, msg
    assert _rel_err(out, ref) < 2e-2
    assert _rel_err(out, ops.paged_attention_ref(q, kc, vc, bt, sl, qs, scale)) < 2e-2
    return w


def test_noalloc_leftovers_head_dim_64_and_prefill_tiling(cuda_device):
    """Two calls with the same token count and split factor: the first fills every split of
    the shared array, the second has contexts short enough that its upper splits hold no keys
    and must overwrite the first call's partials with empty ones.  Then head_dim 64 and the
    prefill (multi-token query) tiling, which needs no scratch."""
    fn = _lib()
    Hq, Hkv, D = 32, 8, 128
    _check(fn, cuda_device, [4000, 3000, 3500, 2500, 3900, 3100, 2900, 3700], Hq, Hkv, D, splits=16, seed=3)
    _check(fn, cuda_device, [5, 20, 1, 40, 9, 30, 2, 16], Hq, Hkv, D, splits=16, seed=4)
    w = _check(fn, cuda_device, [700, 64, 1300, 9, 2000, 333], 16, 4, 64, splits=8, seed=5)
    assert w.decode
    w = _check(fn, cuda_device, [0, 100, 37], Hq, Hkv, D, q_lens=[50, 20, 90], seed=6)
    assert not w.decode

