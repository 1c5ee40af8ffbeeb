"""Sequence-parallel prefill collectives: fused kernels against the NCCL baseline.

One transformer-layer boundary of SP prefill on each rank (Llama-3-70B shapes per TP shard by
default): the row-parallel ``o_proj`` GEMM, reduce-scatter of its output rows, residual add +
RMSNorm of the local rows, all-gather of the normalized rows and the column-parallel
``gate_up`` GEMM over all tokens.

* fused:    gemm_rs (EPI_BF16_RS) -> sp_norm_push -> gemm_ag (SPFusedComm)
* baseline: gemm_out -> NCCL reduce_scatter -> add_rmsnorm -> NCCL all_gather -> gemm_out

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_sp_fused.py [--tokens 4096]
    python benchmarks/bench_sp_fused.py --single      # one GPU: the fused kernels with every
                                                      # "peer" address local (for ncu captures)

Device-timed with CUDA events, maximum over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from vllm_neuron_b200 import ops  # noqa: E402
from vllm_neuron_b200.ops import linear as L  # noqa: E402
from vllm_neuron_b200.ops._ext import ext  # noqa: E402


class _LocalSP:
    """The SPFusedComm protocol with a world of one: slots, gathered rows and counters in this
    GPU's memory (exercises EPI_BF16_RS, sp_norm_push and the all-gather wait on one GPU)."""

    def __init__(self, T: int, H: int, dev):
        self.T, self.H = T, H
        self.x = torch.zeros(2, T, H, dtype=torch.bfloat16, device=dev)
        self.slots = torch.zeros(2, T, H, dtype=torch.bfloat16, device=dev)
        self.ctr = torch.zeros(2, dtype=torch.int32, device=dev)  # [rs, ag]
        self.rs_calls = self.ag_calls = 0
        self.rs_target = self.ag_target = 0

    def gemm_rs(self, a, w, bn):
        par = self.rs_calls % 2
        self.rs_calls += 1
        ext().gemm_sp(a, w, self.x[0, :1], 5, bn, 0, [], 0, [self.slots[par].data_ptr()],
                      [self.ctr.data_ptr()], self.T, None)
        self.rs_target += -(-self.T // 128) * -(-w.shape[0] // bn)

    def norm_push(self, res, nw):
        par = self.ag_calls % 2
        self.ag_calls += 1
        ext().sp_norm_push(self.slots[(self.rs_calls - 1) % 2].data_ptr(), self.T * self.H, 1,
                           self.ctr.data_ptr(), self.rs_target, res, nw, 1e-5,
                           [self.x[par].data_ptr()], [self.ctr.data_ptr() + 4])
        self.ag_target += self.T
        return self.x[par]

    def gemm_ag(self, x, w, out, bn):
        ext().gemm_sp(x, w, out, L.EPI_BF16, bn, self.ctr.data_ptr() + 4, [self.ag_target], self.T, [], [], 0,
                      None)


def _time(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--attn-cols", type=int, default=None, help="o_proj input columns per rank")
    ap.add_argument("--inter", type=int, default=None, help="gate_up rows per rank")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--single", action="store_true")
    a = ap.parse_args()
    from vllm_neuron_b200.parallel import state as ps

    rank, world = ps.init_distributed(timeout_s=120)
    if world > 1:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dev = torch.device("cuda", torch.cuda.current_device())
    W = 1 if a.single else world
    H, T = a.hidden, a.tokens
    Tl = T // W
    A = a.attn_cols or 8192 // W
    I2 = a.inter or 2 * 28672 // W
    g = torch.Generator(device=dev).manual_seed(rank)
    attn = torch.randn(T, A, device=dev, generator=g).to(torch.bfloat16)
    w_o = (torch.randn(H, A, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w_gu = (torch.randn(I2, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    nw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    res = torch.randn(Tl, H, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(T, I2, dtype=torch.bfloat16, device=dev)
    bn_o = L._pick_bn_wide(T, H, L.num_sms(dev))
    bn_g = L._pick_bn_wide(T, I2, L.num_sms(dev))
    row = {"tokens": T, "hidden": H, "o_cols": A, "gate_up_rows": I2, "world": W}
    if W == 1:
        sp = _LocalSP(T, H, dev)

        def fused():
            sp.gemm_rs(attn, w_o, bn_o)
            x = sp.norm_push(res, nw)
            sp.gemm_ag(x, w_gu, out, bn_g)
    else:
        st = ps.initialize_parallel_state(ps.ParallelConfig(world_size=world, tensor_parallel_size=world))
        from vllm_neuron_b200.parallel.fused import SPFusedComm

        spc = SPFusedComm(st.tp, H, T, dev, st.cpu)
        h = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        h_l = torch.empty(Tl, H, dtype=torch.bfloat16, device=dev)
        x_l = torch.empty(Tl, H, dtype=torch.bfloat16, device=dev)
        x_all = torch.empty(T, H, dtype=torch.bfloat16, device=dev)

        def fused():
            spc.gemm_rs(attn, w_o, bn_o)
            x = spc.norm_push(res, nw, 1e-5, reduce=True)
            spc.gemm_ag(x, w_gu, out, L.EPI_BF16, bn_g)

        def baseline():
            L.gemm_out(attn, w_o, out=h)
            dist.reduce_scatter_tensor(h_l, h, group=st.tp.group)
            ops.add_rmsnorm(h_l, res, nw, 1e-5, out=x_l)
            dist.all_gather_into_tensor(x_all, x_l, group=st.tp.group)
            L.gemm_out(x_all, w_gu, out=out)

        row["baseline_ms"] = _time(baseline, a.iters, a.warmup)
    ext().reset_status()
    row["fused_ms"] = _time(fused, a.iters, a.warmup)
    torch.cuda.synchronize()
    row["device_status"] = int(ext().read_status())
    flops = 2.0 * T * A * H + 2.0 * T * H * I2
    row["fused_tflops"] = flops / (row["fused_ms"] * 1e9)
    if world > 1:
        for k in ("fused_ms", "baseline_ms"):
            t = torch.tensor([row[k]], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            row[k] = float(t)
        spc.close()
    if rank == 0:
        print(json.dumps(row), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
