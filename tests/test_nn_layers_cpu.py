"""TP layers (vllm_neuron_b200.nn) on CPU: single rank against torch, and 2 gloo ranks whose
sharded results must equal the unsharded layer."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vllm_neuron_b200 import nn as N
from vllm_neuron_b200.parallel.comm import SINGLE, GroupComm


def test_rejection_sampler_greedy():
    tgt = torch.tensor([[5, 6, 7, 8], [5, 9, 7, 8], [1, 2, 3, 4]])
    drf = torch.tensor([[5, 6, 7], [5, 6, 7], [9, 2, 3]])
    out = N.rejection_sampler(tgt, drf)
    assert out.tolist() == [[5, 6, 7, 8], [5, 9, -1, -1], [1, -1, -1, -1]]
    out2 = N.rejection_sampler(tgt, drf, num_drafts=torch.tensor([1, 3, 3]))
    assert out2[0].tolist() == [5, 6, -1, -1]


def test_single_rank_layers():
    torch.manual_seed(0)
    x = torch.randn(5, 64)
    col = N.ColumnParallelLinear(64, 96, bias=True, dtype=torch.float32)
    w, b = torch.randn(96, 64), torch.randn(96)
    col.load_full_weight(w, b)
    assert torch.allclose(col(x), x @ w.t() + b, atol=1e-4)
    row = N.RowParallelLinear(64, 32, bias=True, dtype=torch.float32)
    w2, b2 = torch.randn(32, 64), torch.randn(32)
    row.load_full_weight(w2, b2)
    assert torch.allclose(row(x), x @ w2.t() + b2, atol=1e-4)
    emb = N.VocabParallelEmbedding(100, 16, dtype=torch.float32)
    t = torch.randn(100, 16)
    emb.load_full_weight(t)
    ids = torch.tensor([0, 5, 99])
    assert torch.equal(emb(ids), t[ids])
    s = N.Sampler()
    lg = torch.randn(3, 50)
    z = torch.zeros(3)
    tok = s(lg, z, torch.zeros(3, dtype=torch.int32), torch.ones(3), torch.zeros(3, dtype=torch.int64),
            torch.zeros(3, dtype=torch.int32))
    assert tok.tolist() == lg.argmax(-1).tolist()


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = GroupComm(dist.group.WORLD)
    g = torch.Generator().manual_seed(0)
    H, Hq, Hkv, D, I, V = 64, 4, 2, 16, 128, 100
    x = torch.randn(6, H, generator=g)
    wqkv = torch.randn((Hq + 2 * Hkv) * D, H, generator=g)
    wo = torch.randn(H, Hq * D, generator=g)
    wg, wu = torch.randn(I, H, generator=g), torch.randn(I, H, generator=g)
    wd = torch.randn(H, I, generator=g)
    table = torch.randn(V, H, generator=g)
    f32 = dict(dtype=torch.float32)
    qkv = N.QKVParallelLinear(H, D, Hq, Hkv, comm=comm, **f32)
    qkv.load_full_weight(wqkv)
    o = N.RowParallelLinear(Hq * D, H, comm=comm, **f32)
    o.load_full_weight(wo)
    gu = N.MergedColumnParallelLinear(H, [I, I], comm=comm, **f32)
    gu.load_full_weight(torch.cat([wg, wu]))
    dn = N.RowParallelLinear(I, H, comm=comm, reduce="scatter", **f32)
    dn.load_full_weight(wd)
    emb = N.VocabParallelEmbedding(V, H, comm=comm, **f32)
    emb.load_full_weight(table)
    ed = N.EmbedDimShardedEmbedding(V, H, comm=comm, **f32)
    ed.load_full_weight(table)
    ids = torch.tensor([0, 7, 50, 99, 3, 64])
    res = {}
    y = qkv(x)  # [q_r | k_r | v_r]
    qd = Hq // world * D
    q_all = comm.all_gather(y[:, :qd].contiguous(), dim=-1)
    res["q"] = torch.allclose(q_all, x @ wqkv[:Hq * D].t(), atol=1e-3)
    res["o"] = torch.allclose(o(q_all[:, rank * qd:(rank + 1) * qd].contiguous()), q_all @ wo.t(), atol=1e-2)
    h = gu(x)
    Il = I // world
    act = torch.nn.functional.silu(h[:, :Il]) * h[:, Il:]
    full_act = torch.nn.functional.silu(x @ wg.t()) * (x @ wu.t())
    y2 = dn(act.contiguous())
    res["mlp_rs"] = torch.allclose(y2, (full_act @ wd.t()).chunk(world, 0)[rank], atol=1e-2)
    res["emb"] = torch.allclose(emb(ids), table[ids])
    res["emb_dim"] = torch.allclose(ed(ids), table[ids])
    q.put((rank, res))
    dist.destroy_process_group()


def test_two_rank_layers_gloo():
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, res in out:
        assert all(res.values()), (rank, res)
