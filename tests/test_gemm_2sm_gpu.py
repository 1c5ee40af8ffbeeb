"""Two-SM (cta_group::2) tcgen05 GEMM against an fp32 oracle.

The CTA-pair kernel serves the dense bf16 prefill shapes (EPI_BF16 and the fused SwiGLU
epilogue, M >= 512).  Covers full tiles, ragged M and N edges (zero-filled rows of the odd CTA,
masked stores), K not a multiple of the 64-element k-block, and agreement with the single-SM
kernel on the same operands.
"""
import pytest
import torch

from vllm_neuron_b200.ops import linear as L
from vllm_neuron_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.fixture
def two_sm():
    e = ext()
    prev = e.gemm_2sm_enabled()
    e.gemm_2sm_set(True)
    yield e
    e.gemm_2sm_set(prev)


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (1000, 6144, 4096), (777, 1000, 4136),
                                   (8192, 4096, 1024), (2304, 768, 4096)])
def test_gemm_2sm_bf16(cuda_device, two_sm, M, N, K):
    g = torch.Generator(device=cuda_device).manual_seed(M + N + K)
    x = torch.randn(M, K, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    out = torch.full((M, N), float("nan"), device=cuda_device, dtype=torch.bfloat16)
    two_sm.gemm(x, w, out, L.EPI_BF16, 256, 1, 0, 0)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    assert not torch.isnan(out).any()
    assert _rel(out, ref) < 1e-2
    # the single-SM kernel on the same operands: same fp32 sums up to the bf16 rounding
    two_sm.gemm_2sm_set(False)
    out1 = torch.empty_like(out)
    two_sm.gemm(x, w, out1, L.EPI_BF16, 256, 1, 0, 0)
    torch.cuda.synchronize()
    two_sm.gemm_2sm_set(True)
    assert _rel(out, out1) < 5e-3


@pytest.mark.parametrize("M,I,K", [(512, 14336, 4096), (1300, 1792, 4096)])
def test_gemm_2sm_silu(cuda_device, two_sm, M, I, K):
    g = torch.Generator(device=cuda_device).manual_seed(M + I)
    x = torch.randn(M, K, device=cuda_device, generator=g).to(torch.bfloat16)
    gate = (torch.randn(I, K, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    up = (torch.randn(I, K, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
    w = L.interleave_gate_up(gate, up)
    out = L.gemm_silu(x, w)
    torch.cuda.synchronize()
    ref = torch.nn.functional.silu(x.float() @ gate.float().t()) * (x.float() @ up.float().t())
    assert _rel(out, ref) < 1e-2


def test_gemm_2sm_repeated_and_status(cuda_device, two_sm):
    """Back-to-back launches (PDL chaining of the cluster kernel) leave no error status."""
    x = torch.randn(4096, 4096, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(6144, 4096, device=cuda_device) * 0.05).to(torch.bfloat16)
    out = torch.empty(4096, 6144, device=cuda_device, dtype=torch.bfloat16)
    for _ in range(20):
        two_sm.gemm(x, w, out, L.EPI_BF16, 256, 1, 0, 0)
    torch.cuda.synchronize()
    assert int(two_sm.read_status()) == 0
    ref = x[:256].float() @ w.float().t()
    assert _rel(out[:256], ref) < 1e-2
