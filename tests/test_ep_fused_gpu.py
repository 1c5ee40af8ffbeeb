"""Device-side expert-parallel exchange (csrc/comm/ep_fused.cu) on two GPUs.

Each rank holds different tokens and half of the experts.  The four-kernel exchange (dispatch
into the owners' receive buffers, receive, expert pipeline on the static row bound, return into
the token owners' combine slots, combine) must give every token the weighted sum of its top-k
experts, as computed locally from the full expert set with the fp32 oracle -- over several
calls with changing token counts (including a rank with no tokens) and when the whole exchange
is replayed from a CUDA graph.  Skipped unless two CUDA devices are visible.
"""
import os
import socket
import subprocess
import sys
import tempfile

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r'''
import os, sys, torch
sys.path.insert(0, sys.argv[1])
import torch.distributed as dist
from vllm_neuron_b200.ops import moe as M
from vllm_neuron_b200.ops._ext import ext
from vllm_neuron_b200.parallel.ep_fused import EPFusedExchange

rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", device_id=dev)
cpu = dist.new_group(backend="gloo")
E, k, H, I, cap = 8, 2, 1024, 512, 96
e_local = E // world
g = torch.Generator().manual_seed(0)  # same full expert set on every rank
w_gu_all = (torch.randn(E, 2 * I, H, generator=g) * 0.03).to(torch.bfloat16)
w_dn_all = (torch.randn(E, H, I, generator=g) * 0.03).to(torch.bfloat16)
e0 = rank * e_local
w_gu = w_gu_all[e0:e0 + e_local].to(dev).contiguous()
w_dn = w_dn_all[e0:e0 + e_local].to(dev).contiguous()
ex = EPFusedExchange(dist.group.WORLD, rank, world, E, k, H, cap, dev, cpu)
ws = M.MoEWorkspace.create(ex.rows_cap, k, E, e_local, H, I, dev)
y = torch.zeros(ex.rows_cap, H, dtype=torch.bfloat16, device=dev)
out = torch.zeros(cap, H, dtype=torch.bfloat16, device=dev)

def step(x, ids, w):
    ex.dispatch(x, ids, w)
    rows, rids, rw = ex.recv()
    M._experts_cuda(rows, rids, rw, w_gu, w_dn, k, None, None, M.ACT_SILU, 1.702, 7.0, e0, ws, y,
                    None, None, None, None, 0)
    ex.ret(y)
    return ex.combine(out[:x.shape[0]])

def batch(T, seed):
    gg = torch.Generator().manual_seed(1000 * seed + rank)
    x = (torch.randn(T, H, generator=gg) * 0.5).to(torch.bfloat16).to(dev)
    ids = torch.stack([torch.randperm(E, generator=gg)[:k] for _ in range(T)]).to(torch.int32).to(dev) \
        if T else torch.zeros(0, k, dtype=torch.int32, device=dev)
    w = torch.rand(T, k, generator=gg).to(dev)
    return x, ids, w

def check(x, ids, w, got, tag):
    if x.shape[0] == 0:
        return
    ref = M.experts_ref(x.float().cpu(), ids.cpu(), w.cpu(), w_gu_all.float(), w_dn_all.float())
    rel = float((got.float().cpu() - ref).norm() / ref.norm())
    assert rel < 2e-2, (tag, rank, rel)

sizes = [[37, 64], [0, 5], [96, 1], [64, 64]]
for i, ts in enumerate(sizes):
    x, ids, w = batch(ts[rank], i)
    got = step(x, ids, w)
    torch.cuda.synchronize()
    assert ext().read_status() == 0, ("status", i)
    check(x, ids, w, got, f"eager{i}")
# the whole exchange replayed from a CUDA graph (static shapes, device-side call counter)
x, ids, w = batch(48, 99)
s = torch.cuda.Stream()
with torch.cuda.stream(s):
    step(x, ids, w)
torch.cuda.synchronize()
dist.barrier()
gr = torch.cuda.CUDAGraph()
with torch.cuda.graph(gr, stream=s):
    got = step(x, ids, w)
for rep in range(3):
    x2, ids2, w2 = batch(48, 200 + rep)
    x.copy_(x2); ids.copy_(ids2); w.copy_(w2)
    gr.replay()
    torch.cuda.synchronize()
    assert ext().read_status() == 0, ("status graph", rep)
    check(x, ids, w, got, f"graph{rep}")
dist.barrier()
del gr
ex.close()
print("EP_OK", rank, flush=True)
dist.barrier()
os._exit(0)
'''


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_ep_fused_exchange_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tempfile.mktemp(suffix=".py")
    with open(script, "w") as f:
        f.write(WORKER)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", script, ROOT]
    r = subprocess.run(["timeout", "-k", "30", "240"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("EP_OK") == 2, r.stdout[-2000:]
