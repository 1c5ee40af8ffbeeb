"""Gated DeltaNet kernels on the GPU against the fp32 oracles: varlen batches with fresh and
continuing sequences (state cache), decode steps, GQA-style key/value head ratios."""
import pytest
import torch

from vllm_neuron_b200.ops import deltanet as DN
from vllm_neuron_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _status(cuda_device):
    torch.manual_seed(0)
    ext().reset_status()
    yield
    torch.cuda.synchronize()
    assert ext().read_status() == 0


def _batch(q_lens, ctx, dev):
    qs = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32, device=dev)
    sl = torch.tensor([c + q for c, q in zip(ctx, q_lens)], dtype=torch.int32, device=dev)
    slots = torch.tensor([3 * i + 1 for i in range(len(q_lens))], dtype=torch.int32, device=dev)
    return qs, sl, slots


@pytest.mark.parametrize("K", [4, 2])
def test_causal_conv1d(cuda_device, K):
    C = 384
    q_lens, ctx = [1, 37, 5, 200, 1], [10, 0, 3, 0, 0]
    qs, sl, slots = _batch(q_lens, ctx, cuda_device)
    T = sum(q_lens)
    x = torch.randn(T, C, device=cuda_device).to(torch.bfloat16)
    w = torch.randn(C, K, device=cuda_device).to(torch.bfloat16) * 0.5
    state = torch.randn(20, C, K - 1, device=cuda_device).to(torch.bfloat16)
    st_ref = state.float().cpu().clone()
    out = torch.empty(T, C, device=cuda_device, dtype=torch.bfloat16)
    DN.causal_conv1d(x, w, qs, sl, slots, state, out)
    ref = DN.causal_conv1d_ref(x.cpu().float(), w.cpu().float(), qs.cpu(), sl.cpu(), slots.cpu(), st_ref)
    assert _rel_err(out.cpu(), ref) < 1e-2
    assert _rel_err(state.cpu(), st_ref) < 1e-2


@pytest.mark.parametrize("mode", ["recurrent", "chunked"])
@pytest.mark.parametrize("Hk,Hv", [(2, 4), (4, 4)])
def test_gated_delta_rule(cuda_device, Hk, Hv, mode):
    dk = dv = 128
    q_lens, ctx = [1, 64, 7, 130, 1, 1], [20, 0, 5, 0, 0, 300]
    qs, sl, slots = _batch(q_lens, ctx, cuda_device)
    T = sum(q_lens)
    qkv = torch.randn(T, 2 * Hk * dk + Hv * dv, device=cuda_device).to(torch.bfloat16)
    zab = torch.randn(T, Hv * dv + 2 * Hv, device=cuda_device).to(torch.bfloat16)
    z, b, a = zab[:, :Hv * dv], zab[:, Hv * dv:Hv * dv + Hv], zab[:, Hv * dv + Hv:]
    A_log = torch.rand(Hv, device=cuda_device).mul(3).add(0.1).log()
    dt_bias = torch.randn(Hv, device=cuda_device) * 0.5
    nw = (1 + 0.1 * torch.randn(dv, device=cuda_device)).to(torch.bfloat16)
    state = torch.randn(20, Hv, dk, dv, device=cuda_device) * 0.1
    st_ref = state.cpu().clone()
    out = torch.empty(T, Hv * dv, device=cuda_device, dtype=torch.bfloat16)
    for _ in range(2):  # the second call continues from the updated state
        DN.gated_delta_rule(qkv, z, a, b, A_log, dt_bias, nw, 1e-6, qs, sl, slots, state, out, Hk, Hv,
                            mode=mode)
        ref = DN.gated_delta_rule_ref(qkv.cpu(), z.cpu(), a.cpu(), b.cpu(), A_log.cpu(), dt_bias.cpu(),
                                      nw.cpu(), 1e-6, qs.cpu(), sl.cpu(), slots.cpu(), st_ref, Hk, Hv)
        assert _rel_err(out.cpu(), ref) < 2e-2
        # the chunked form multiplies bf16-rounded unit q / k on the tensor cores
        assert _rel_err(state.cpu(), st_ref) < (1e-3 if mode == "recurrent" else 5e-3)
        sl = sl + torch.tensor(q_lens, dtype=torch.int32, device=cuda_device)


def test_sigmoid_gate_mul(cuda_device):
    x = torch.randn(33, 512, device=cuda_device).to(torch.bfloat16)
    g = torch.randn(33, 1024, device=cuda_device).to(torch.bfloat16)[:, 256:768]
    ref = x.float() * torch.sigmoid(g.float())
    DN.sigmoid_gate_mul(x, g)
    assert _rel_err(x, ref) < 1e-2


def test_gated_delta_rule_chunked_long(cuda_device):
    """Many chunks per sequence (state carried across 16 chunks) against the recurrent kernel,
    with a continuing sequence and a ragged last chunk; Qwen3.6-like head ratio."""
    Hk, Hv, dk = 4, 8, 128
    q_lens, ctx = [1000, 777, 1], [0, 50, 9]
    qs, sl, slots = _batch(q_lens, ctx, cuda_device)
    T = sum(q_lens)
    qkv = torch.randn(T, 2 * Hk * dk + Hv * dk, device=cuda_device).to(torch.bfloat16)
    zab = torch.randn(T, Hv * dk + 2 * Hv, device=cuda_device).to(torch.bfloat16)
    z, b, a = zab[:, :Hv * dk], zab[:, Hv * dk:Hv * dk + Hv], zab[:, Hv * dk + Hv:]
    A_log = torch.rand(Hv, device=cuda_device).mul(3).add(0.1).log()
    dt_bias = torch.randn(Hv, device=cuda_device) * 0.5 - 2.0  # slow decays: long memory
    nw = (1 + 0.1 * torch.randn(dk, device=cuda_device)).to(torch.bfloat16)
    state = torch.randn(20, Hv, dk, dk, device=cuda_device) * 0.1
    st_rec = state.clone()
    out = torch.empty(T, Hv * dk, device=cuda_device, dtype=torch.bfloat16)
    out_rec = torch.empty_like(out)
    DN.gated_delta_rule(qkv, z, a, b, A_log, dt_bias, nw, 1e-6, qs, sl, slots, state, out, Hk, Hv,
                        mode="chunked")
    DN.gated_delta_rule(qkv, z, a, b, A_log, dt_bias, nw, 1e-6, qs, sl, slots, st_rec, out_rec, Hk,
                        Hv, mode="recurrent")
    assert _rel_err(out, out_rec) < 2e-2
    assert _rel_err(state, st_rec) < 1e-2
