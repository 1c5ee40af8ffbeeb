"""Decode context parallelism on one B200: the ranks of a replica set are emulated by running
the attention kernel once per rank over that rank's token shard (partial output + LSE with the
DCP causal mapping), then the split-merge kernel combines all partials; the result must match
the fp32 oracle over the whole sequence."""
import numpy as np
import pytest
import torch

from tests.test_dcp_cpu import full_cache, shard_cache
from vllm_neuron_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("q_lens,seq_lens,dcp,splits", [
    ([1] * 6, [37, 640, 5, 1000, 129, 64], 2, None),   # decode (TMA decode kernel)
    ([1] * 3, [300, 17, 2049], 4, None),
    ([2, 3, 1], [40, 300, 77], 2, None),                # multi-token decode rows (drafts)
    ([70, 1, 9], [70, 500, 200], 2, 1),                 # prefill chunks + decode (generic kernel)
    ([130, 5], [400, 260], 4, 1),
])
def test_dcp_attention_matches_full(q_lens, seq_lens, dcp, splits):
    torch.manual_seed(1)
    dev = "cuda"
    bs, Hkv, D = 16, 1, 128
    G_local = 2                       # query heads per rank
    Hq = G_local * dcp                # gathered over the replica set
    B = len(seq_lens)
    Lmax = max(seq_lens)
    bps = (Lmax + bs - 1) // bs
    k_full = torch.randn(B, Hkv, Lmax, D) * 0.5
    v_full = torch.randn(B, Hkv, Lmax, D)
    T = sum(q_lens)
    q = (torch.randn(T, Hq, D) * 0.5).to(torch.bfloat16)
    qs = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    q_start = torch.tensor(qs, device=dev)
    sl = torch.tensor(seq_lens, dtype=torch.int32, device=dev)
    scale = D ** -0.5

    kc, vc, bt_full = full_cache(k_full.bfloat16().float(), v_full.bfloat16().float(), bs, bps)
    want = ops.paged_attention_ref(q.float().to(dev), kc.to(dev), vc.to(dev), bt_full.to(dev), sl,
                                   q_start, scale)

    caches, bt = shard_cache(k_full, v_full, seq_lens, bs, dcp, bps)
    bt = bt.to(dev)
    parts_o, parts_l = [], []
    for r, (kcr, vcr, local) in enumerate(caches):
        w = ops.build_work(np.asarray(q_lens), np.asarray(local), Hq // Hkv, Hkv, 148,
                           head_dim=D)
        ns = splits or w.num_splits
        po = torch.empty(ns, T, Hq, D, device=dev)
        pl = torch.empty(ns, T, Hq, device=dev)
        ops.paged_attention_partial(q.to(dev), kcr.bfloat16().to(dev), vcr.bfloat16().to(dev), bt,
                                    torch.tensor(local, dtype=torch.int32, device=dev), q_start,
                                    torch.from_numpy(w.work).to(dev), w.decode, ns, scale, po, pl,
                                    dcp_seq_lens=sl, dcp_size=dcp, dcp_rank=r)
        parts_o.append(po)
        parts_l.append(pl)
    got = ops.attn_combine(torch.cat(parts_o), torch.cat(parts_l))
    torch.cuda.synchronize()
    err = (got.float() - want).abs().max().item()
    assert err < 2e-2, err
