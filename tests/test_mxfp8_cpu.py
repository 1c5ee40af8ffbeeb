"""MXFP8 host side: the e8m0 exponent rule (smallest power of two that keeps every value of a
32-group within e4m3's 448), exact dequantization, the scale-atom layout of the block-scaled
GEMM, and the CPU path of the projections (the fp32 oracle)."""
import torch

from vllm_neuron_b200.ops import linear as L


def test_exponent_rule():
    amax = torch.tensor([0.0, 448.0, 448.5, 1.0, 896.0, 1e-30, 3e38])
    e = L.mx8_exponents(amax)
    assert e.tolist()[:5] == [0, 0, 1, -8, 1]
    for a, k in zip(amax.tolist(), e.tolist()):
        if a > 0 and -127 < k < 127:
            assert a <= 448 * 2.0 ** k and a > 448 * 2.0 ** (k - 1)


def test_quantize_round_trip_and_no_saturation():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(9, 256, generator=g) * torch.exp(torch.randn(9, 8, generator=g) * 3).repeat_interleave(32, 1)
    q, s = L.quantize_mx8(x)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (9, 8)
    assert torch.isfinite(q.float()).all() and q.float().abs().max() <= 448
    d = L.dequantize_mx8(q, s)
    assert float((d - x).norm() / x.norm()) < 0.04
    # power-of-two scaling: the dequantized values are exactly representable again
    q2, s2 = L.quantize_mx8(d)
    assert torch.equal(L.dequantize_mx8(q2, s2), d)


def test_atom_layout():
    s = torch.arange(300 * 8, dtype=torch.int32).remainder(251).to(torch.uint8).view(300, 8)
    a = L.mx8_atoms(s)
    assert a.shape == (3, 2, 512)
    for r in (0, 31, 32, 77, 127, 128, 299):
        for kb in (0, 1):
            off = (r % 32) * 16 + ((r % 128) // 32) * 4
            assert a[r // 128, kb, off:off + 4].tolist() == s[r, kb * 4:kb * 4 + 4].tolist()
    assert int(a[2, :, :].view(-1).sum()) > 0 and a.view(3, -1)[2].numel() == 1024


def test_cpu_projection_paths():
    g = torch.Generator().manual_seed(1)
    w = L.MXFP8Weight.from_weight(torch.randn(256, 256, generator=g) * 0.05)
    x = torch.randn(5, 256, generator=g)
    ref = L._mx8_ref(x, w)
    out = L.gemm_out(x, w)
    assert torch.allclose(out.float(), ref, atol=1e-4, rtol=1e-4)
    acc = torch.zeros(5, 256)
    L.gemm_accumulate(x, w, acc)
    assert torch.allclose(acc, ref, atol=1e-4, rtol=1e-4)
    gu = L.MXFP8Weight.from_weight(torch.randn(2 * L.SILU_BLOCK, 256, generator=g) * 0.05)
    y = L.gemm_silu(x, gu)  # bf16 output
    assert torch.allclose(y.float(), L.silu_mul_ref(L._mx8_ref(x, gu), L.SILU_BLOCK), atol=1e-2, rtol=1e-2)


def _mx_checkpoint():
    """The tiny Llama in the LLM-Compressor MXFP8 layout: e4m3 projection weights with a uint8
    ``weight_scale`` [N, K / 32] (e8m0), no input scales."""
    import os
    import tempfile

    from safetensors.torch import load_file, save_file

    from tests._tiny import tiny_llama_checkpoint

    src, _ = tiny_llama_checkpoint()
    d = tempfile.mkdtemp(prefix="tiny_llama_mxfp8_")
    for f in os.listdir(src):
        if not f.endswith(".safetensors"):
            os.system(f"cp '{os.path.join(src, f)}' '{d}'")
    sd = load_file(os.path.join(src, "model.safetensors"))
    out, deq = {}, {}
    for k, v in sd.items():
        if k.endswith("_proj.weight"):
            q, s = L.quantize_mx8(v.float())
            out[k], out[k.replace(".weight", ".weight_scale")] = q, s
            deq[k] = L.dequantize_mx8(q, s)
        else:
            out[k] = deq[k] = v
    save_file(out, os.path.join(d, "model.safetensors"))
    ref = tempfile.mkdtemp(prefix="tiny_llama_mxref_")
    for f in os.listdir(src):
        if not f.endswith(".safetensors"):
            os.system(f"cp '{os.path.join(src, f)}' '{ref}'")
    save_file({k: v.contiguous() for k, v in deq.items()}, os.path.join(ref, "model.safetensors"))
    return d, ref


def test_mxfp8_checkpoint_loads_exactly_and_serves_mx():
    """An MXFP8 checkpoint reads as its exact dequantized values; with quantization='mxfp8' the
    projections become MXFP8 weights (the CPU path runs the W8A8 oracle) and their values equal
    the checkpoint's."""
    from vllm_neuron_b200.entrypoints import LLM
    from tests._tiny import random_prompts

    kw = dict(device="cpu", dtype="float32", max_num_seqs=4, max_model_len=128, num_gpu_blocks=64,
              skip_tokenizer_init=True)
    d, ref = _mx_checkpoint()
    prompts = random_prompts(n=2, length=16, seed=4)
    exact = LLM(ref, **kw).engine.prompt_logits(prompts)
    plain = LLM(d, **kw)
    assert torch.equal(plain.engine.prompt_logits(prompts), exact)
    mx = LLM(d, additional_config={"neuron_config": {"quantization": "mxfp8"}}, **kw)
    m = mx.engine.model
    assert m.mx_linears == 2 * 4 and isinstance(m.layers[0].qkv, L.MXFP8Weight)
    assert torch.equal(m.layers[0].o.dequant(), plain.engine.model.layers[0].o.float())
    got = mx.engine.prompt_logits(prompts)
    rel = float((got - exact).norm() / exact.norm())
    assert rel < 0.05, rel  # the activations' MXFP8 rounding only


def test_mxfp4_reencodes_losslessly_with_padding():
    from vllm_neuron_b200.models.gpt_oss import _quant_experts

    g = torch.Generator().manual_seed(5)
    b, s = _quant_experts(torch.randn(3, 96, 320, generator=g) * 0.1)
    w4 = L.MXFP4Weight.from_blocks(b, s)
    w8 = L.MXFP8Weight.from_mxfp4(w4, k_pad=384, n_pad=128)
    assert w8.q.shape == (3, 128, 384) and w8.sf.shape == (3, 3, 512)
    d8 = w8.dequant()
    assert torch.equal(d8[:, :96, :320], w4.dequant_bf16_ref().float())
    assert d8[:, 96:].abs().sum() == 0 and d8[:, :, 320:].abs().sum() == 0
