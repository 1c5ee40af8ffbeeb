"""Dense projections on the tcgen05 GEMM (csrc/gemm/gemm_sm100.cu).

Weights are stored ``[out_features, in_features]`` (K-contiguous, as checkpoints store them),
activations ``[tokens, in_features]``.  Two regimes:

* ``tokens > SKINNY_MAX`` (prefill / mixed batches): ``out = x @ w^T`` with 128 x BN tiles,
  BN picked to minimise the persistent-wave makespan over the SMs.
* ``tokens <= SKINNY_MAX`` (decode): operands are swapped so the weight rows fill the
  128-row MMA dimension and the tokens become a narrow N tile (16..128).  The K loop is
  split until the grid covers the SMs, and the partial sums are reduced in fp32 into an
  accumulation buffer that the consumer kernel (add_rmsnorm / rope_kv_write / silu_mul)
  reads and clears.

Reference counterparts: ``ColumnParallelLinear`` / ``RowParallelLinear``
(vllm_neuron/nn/cpl.py:27, nn/rpl.py:23) and the NKI projection kernels they feed
(functional/attention/o_proj.py:124, functional/mlp.py:65).
"""
from __future__ import annotations

import math

import torch

from ._ext import ext

EPI_BF16 = 0
EPI_BF16_T = 1
EPI_F32_RED = 2
EPI_F32_RED_T = 3
EPI_SILU_BF16 = 4

FP8_MAX = 448.0


class FP8Weight:
    """Static per-tensor FP8 (e4m3) weight ``[N, K]`` of a linear layer, with its weight scale and
    the static scale of its input activations (W8A8, as in ModelOpt / compressed-tensors static
    FP8 checkpoints): ``y = (quant(x / in_scale) @ q^T) * in_scale * w_scale``.  The GEMM functions
    below accept it wherever they take a bf16 weight.  Reference: the ModelOpt static FP8 path,
    vllm_neuron/model/llama3/quantization.py:39-310."""

    def __init__(self, q: torch.Tensor, w_scale: float, in_scale: float):
        assert q.dtype == torch.float8_e4m3fn and q.dim() == 2
        self.q = q
        self.w_scale = float(w_scale)
        self.in_scale = float(in_scale)

    @classmethod
    def from_weight(cls, w: torch.Tensor, w_scale: float | None = None, in_scale: float = 1.0 / 32) -> "FP8Weight":
        """Quantize ``w`` with ``w_scale`` (default: amax / 448)."""
        if w_scale is None:
            w_scale = max(float(w.detach().abs().max()), 1e-12) / FP8_MAX
        return cls(quantize_fp8(w.detach(), w_scale), w_scale, in_scale)

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device

    def dequant(self) -> torch.Tensor:
        return self.q.float() * self.w_scale


class BlockFP8Weight:
    """Block-scaled FP8 weight ``[N, K]`` (or stacked experts ``[E, N, K]``): e4m3 values ``q``
    and one fp32 scale per 128 x 128 block, ``scales [ceil(rows / 128), ceil(K / 128)]`` over the
    (stacked) rows, true weight = ``q * scale`` -- the layout of DeepSeek / Qwen FP8 checkpoints
    (``weight`` + ``weight_scale_inv``).  Served W8A16: the GEMM streams the fp8 bytes and widens
    each weight tile in shared memory with its block scale (bf16 activations, fp32 accumulation),
    so decode reads half the bytes of bf16 weights.  Expert stacks need rows per expert to be a
    multiple of 128."""

    BLOCK = 128

    def __init__(self, q: torch.Tensor, scales: torch.Tensor):
        assert q.dtype == torch.float8_e4m3fn and q.dim() in (2, 3)
        rows = q.shape[0] * q.shape[1] if q.dim() == 3 else q.shape[0]
        assert scales.dtype == torch.float32 and scales.dim() == 2
        assert scales.shape[0] == -(-rows // self.BLOCK) and scales.shape[1] == -(-q.shape[-1] // self.BLOCK)
        self.q = q
        self.scales = scales

    @classmethod
    def from_weight(cls, w: torch.Tensor) -> "BlockFP8Weight":
        """Quantize ``w`` per 128 x 128 block with scale ``amax / 448``."""
        w = w.detach()
        shp = w.shape
        w2 = w.reshape(-1, shp[-1])
        N, K = w2.shape
        B = cls.BLOCK
        nb, kb = -(-N // B), -(-K // B)
        pad = torch.zeros(nb * B, kb * B, dtype=torch.float32, device=w.device)
        pad[:N, :K] = w2.float()
        blk = pad.view(nb, B, kb, B)
        sc = (blk.abs().amax(dim=(1, 3)) / FP8_MAX).clamp_min(1e-12)
        q = (blk / sc[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).view(nb * B, kb * B)[:N, :K]
        return cls(q.to(torch.float8_e4m3fn).reshape(shp).contiguous(), sc.contiguous())

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device

    def dequant(self, dtype=torch.float32) -> torch.Tensor:
        """``q * scale`` (the fp32 oracle; the kernels round each product to bf16)."""
        q2 = self.q.reshape(-1, self.q.shape[-1]).float()
        B = self.BLOCK
        s = self.scales.repeat_interleave(B, 0)[: q2.shape[0]].repeat_interleave(B, 1)[:, : q2.shape[1]]
        return (q2 * s).to(dtype).reshape(self.q.shape)

    def dequant_bf16_ref(self) -> torch.Tensor:
        """``bf16(q * scale)``: exactly the operand the tensor cores multiply."""
        return self.dequant(torch.float32).to(torch.bfloat16)


def mx8_exponents(amax: torch.Tensor) -> torch.Tensor:
    """Unbiased e8m0 exponents of MXFP8 groups: the smallest ``e`` with ``amax <= 448 * 2^e``
    (0 for all-zero groups), clamped to the e8m0 range [-127, 127].  Read from the fp32 bits so
    that every device agrees exactly."""
    bits = amax.float().contiguous().view(torch.int32)
    e = ((bits >> 23) & 0xFF) - 135 + ((bits & 0x7FFFFF) > 0x600000).to(torch.int32)
    e = torch.where(amax == 0, torch.zeros_like(e), e)
    return e.clamp(-127, 127)


def _pow2(e: torch.Tensor) -> torch.Tensor:
    """Exact fp32 ``2^e`` for integer ``e`` in [-127, 127] (the e8m0 range)."""
    bits = torch.where(e <= -127, torch.full_like(e, 0x00400000), (e + 127).clamp(1, 254) << 23)
    return bits.to(torch.int32).view(torch.float32)


def quantize_mx8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """OCP MXFP8 of ``x [..., K]`` (K a multiple of 32): e4m3 values and biased e8m0 scales
    ``[..., K / 32]`` (uint8), true value = ``q * 2^(s - 127)``.  Bit-identical to the device
    quantizer (power-of-two scaling, then round-to-nearest-even e4m3)."""
    *lead, K = x.shape
    g = x.float().reshape(-1, K // 32, 32)
    e = mx8_exponents(g.abs().amax(-1))
    q = (g * _pow2(-e)[..., None]).to(torch.float8_e4m3fn)
    return q.reshape(*lead, K), (e + 127).to(torch.uint8).reshape(*lead, K // 32)


def mx8_atoms(scales: torch.Tensor, rows: int | None = None) -> torch.Tensor:
    """Linear e8m0 scales ``[R, K / 32]`` -> the block-scaled GEMM's 512-byte atoms
    ``[ceil(R / 128), K / 128, 512]``: atom (row block, 128-wide k block) holds row r's four
    group scales at ``(r % 32) * 16 + ((r / 32) % 4) * 4``; rows past ``R`` are zero."""
    R, G = scales.shape
    assert G % 4 == 0, "K must be a multiple of 128"
    nb = -(-(rows or R) // 128)
    pad = torch.zeros(nb * 128, G, dtype=torch.uint8, device=scales.device)
    pad[:R] = scales
    # r = rb * 128 + r4 * 32 + r32, g = kb * 4 + j  ->  [rb, kb, r32, r4, j]
    return pad.view(nb, 4, 32, G // 4, 4).permute(0, 3, 2, 1, 4).contiguous().view(nb, G // 4, 512)


def dequantize_mx8(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 ``q * 2^(s - 127)`` of an MXFP8 tensor."""
    *lead, K = q.shape
    e = scales.to(torch.int32) - 127
    return (q.float().reshape(-1, K // 32, 32) * _pow2(e.reshape(-1, K // 32))[..., None]).reshape(*lead, K)


class MXFP8Weight:
    """MXFP8 weight ``[N, K]`` (OCP microscaling: e4m3 values, one e8m0 scale per 32 elements
    along K), the format of LLM-Compressor MXFP8 checkpoints (``weight`` F8_E4M3 +
    ``weight_scale`` U8 ``[N, K / 32]``).  Served W8A8 on the block-scaled tensor cores
    (``tcgen05.mma kind::mxf8f6f4.block_scale``): activations are quantized to MXFP8 per token and
    32 elements, both operands stream as bytes and the hardware applies the scales.  K must be a
    multiple of 128."""

    def __init__(self, q: torch.Tensor, scales: torch.Tensor):
        assert q.dtype == torch.float8_e4m3fn and q.dim() in (2, 3) and scales.dtype == torch.uint8
        K = q.shape[-1]
        assert K % 128 == 0 and tuple(scales.shape) == (*q.shape[:-1], K // 32)
        self.q = q.contiguous()
        self.scales = scales.contiguous()
        # expert stacks [E, N, K]: atoms over the stacked rows (N a multiple of 128 for the
        # grouped GEMM, so every expert starts an atom)
        self.sf = mx8_atoms(self.scales.reshape(-1, K // 32))

    @classmethod
    def from_weight(cls, w: torch.Tensor) -> "MXFP8Weight":
        q, s = quantize_mx8(w.detach())
        return cls(q, s)

    @classmethod
    def from_mxfp4(cls, w: "MXFP4Weight", k_pad: int | None = None, n_pad: int | None = None) -> "MXFP8Weight":
        """Lossless re-encoding of an MXFP4 weight (every e2m1 value is an e4m3 value; the e8m0
        scales carry over), optionally padded with zeros to ``k_pad`` columns and ``n_pad`` rows
        (the grouped block-scaled GEMM wants K in 128s and 128-row experts)."""
        lut = torch.tensor(FP4_VALUES, dtype=torch.float32, device=w.q.device)
        lo, hi = (w.q & 0xF).long(), (w.q >> 4).long()
        vals = torch.stack([lut[lo], lut[hi]], dim=-1).flatten(-2)  # [..., N, K]
        *lead, N, K = vals.shape
        kp, np_ = k_pad or K, n_pad or N
        assert kp >= K and kp % 128 == 0 and np_ >= N
        q = torch.zeros(*lead, np_, kp, dtype=torch.float8_e4m3fn, device=w.q.device)
        q[..., :N, :K] = vals.to(torch.float8_e4m3fn)
        sc = torch.full((*lead, np_, kp // 32), 127, dtype=torch.uint8, device=w.q.device)
        sc[..., :N, :K // 32] = w.scales
        return cls(q, sc)

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device

    def dequant(self, dtype=torch.float32) -> torch.Tensor:
        return dequantize_mx8(self.q, self.scales).to(dtype)

    def __getitem__(self, e: int) -> "MXFP8Weight":
        """Expert ``e`` of a stack."""
        return MXFP8Weight(self.q[e], self.scales[e])

    def dequant_bf16_ref(self) -> torch.Tensor:
        """The weight as bf16 (exact: e4m3 times a power of two)."""
        return self.dequant(torch.float32).to(torch.bfloat16)


class MX8Activations:
    """Reusable MXFP8 activation buffers of one projection input: e4m3 ``q [rows, K]`` and the
    scale atoms (zeroed once, so padded rows of the last atom stay finite)."""

    _cache: dict = {}
    _retired: list = []  # outgrown buffers stay alive: CUDA graphs may have captured them

    @classmethod
    def get(cls, rows: int, K: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        key = (str(device), K)
        cur = cls._cache.get(key)
        if cur is None or cur[0].shape[0] < rows:
            if cur is not None:
                cls._retired.append(cur)
            cap = max(rows, 128)
            q = torch.empty(cap, K, dtype=torch.float8_e4m3fn, device=device)
            sf = torch.zeros(-(-cap // 128), K // 128, 512, dtype=torch.uint8, device=device)
            cur = cls._cache[key] = (q, sf)
        return cur[0][:rows], cur[1]

    @classmethod
    def reserve(cls, rows: int, K: int, device):
        """Allocate for ``rows`` up front (before graph capture)."""
        cls.get(rows, K, device)


def mx8_quantize_device(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """MXFP8 of bf16 activations on the GPU into reusable buffers: (q, scale atoms)."""
    M, K = x.shape
    q, sf = MX8Activations.get(M, K, x.device)
    ext().quant_mx8(x, q, sf)
    return q, sf


# e2m1 code points (sign bit 3, exponent bits 2-1, mantissa bit 0)
FP4_VALUES = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


class MXFP4Weight:
    """MXFP4 weight ``[N, K]`` or expert stack ``[E, N, K]`` in the OCP MX layout of GPT-OSS
    checkpoints: ``q [..., N, K / 2]`` uint8 (two e2m1 values per byte, the lower k in the low
    nibble) and ``scales [..., N, K / 32]`` uint8 (e8m0, value ``2 ** (s - 127)``).  Served W4A16 on
    the tcgen05 GEMM: the packed bytes stream from HBM at half a byte per element and each tile is
    widened in shared memory (``e2m1 * scale`` is exact in bf16); bf16 activations, fp32
    accumulation.  K must be a multiple of 64."""

    def __init__(self, q: torch.Tensor, scales: torch.Tensor):
        assert q.dtype == torch.uint8 and scales.dtype == torch.uint8
        assert q.shape[:-1] == scales.shape[:-1] and scales.shape[-1] * 16 == q.shape[-1]
        self.q = q.contiguous()
        self.scales = scales.contiguous()

    @classmethod
    def from_blocks(cls, blocks: torch.Tensor, scales: torch.Tensor) -> "MXFP4Weight":
        """Checkpoint tensors ``blocks [..., K / 32, 16]`` and ``scales [..., K / 32]``."""
        return cls(blocks.reshape(*blocks.shape[:-2], blocks.shape[-2] * 16), scales)

    @property
    def shape(self):
        return (*self.q.shape[:-1], self.q.shape[-1] * 2)

    @property
    def device(self):
        return self.q.device

    def dequant(self, dtype=torch.float32) -> torch.Tensor:
        lut = torch.tensor(FP4_VALUES, dtype=torch.float32, device=self.q.device)
        b = self.q.to(torch.int64)
        v = torch.stack([lut[b & 0x0F], lut[b >> 4]], dim=-1).reshape(*self.q.shape[:-1], -1)
        e = self.scales.to(torch.float32) - 127.0
        v = v.reshape(*v.shape[:-1], -1, 32) * torch.pow(2.0, e)[..., None]
        return v.reshape(self.shape).to(dtype)

    def dequant_bf16_ref(self) -> torch.Tensor:
        return self.dequant(torch.float32).to(torch.bfloat16)


def quantize_fp8(x: torch.Tensor, scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """``satfinite(x / scale)`` as ``torch.float8_e4m3fn`` (the rule of the quant kernels)."""
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    inv = 1.0 / float(scale)
    if x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1 and x.shape[1] % 8 == 0:
        ext().quant_fp8(x, out, inv)
        return out
    out.copy_((x.float() * torch.tensor(inv, dtype=torch.float32)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn))
    return out


def rmsnorm_quant(x: torch.Tensor, w: torch.Tensor, eps: float, scale: float | None = None
                  ) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``rmsnorm(x) * w`` quantized to e4m3: with a static per-tensor ``scale`` (STATIC) or, with
    ``scale=None``, a per-row scale ``max|y| / 448`` returned as fp32 ``[rows]`` (ROW).
    Reference: vllm_neuron/functional/rmsnorm_quant.py:216."""
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    rows = None if scale is not None else torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    if x.is_cuda:
        ext().rmsnorm_quant(x, w, eps, out, 1.0 / scale if scale is not None else 1.0, rows)
        return out, rows
    xf = x.float()
    y = (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps)).to(torch.bfloat16).float() * w.float()
    if scale is None:
        rows = (y.abs().amax(-1) / FP8_MAX).clamp_min(1e-30)
        rows = torch.where(y.abs().amax(-1) > 0, rows, torch.ones_like(rows))
        out.copy_((y / rows[:, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn))
    else:
        out.copy_((y * torch.tensor(1.0 / scale)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn))
    return out, rows


def _fp8_ref(xq: torch.Tensor, w: FP8Weight) -> torch.Tensor:
    return (xq.float() @ w.q.float().t()) * (w.in_scale * w.w_scale)


SKINNY_MAX = 128
SILU_BLOCK = 128  # gate/up interleave block = BN/2 of the fused SwiGLU epilogue

# Library-GEMM mode (``use_cublas_baseline``): the dense bf16 projections run on cuBLAS through
# torch.mm instead of the tcgen05 kernels; everything else (attention, norms, RoPE, sampling)
# stays on this framework's kernels.  This is the same-box NCCL + cuBLAS comparison build.
_LIBRARY_GEMM = False


def set_library_gemm(on: bool) -> None:
    """Route the dense bf16 projections through cuBLAS (``True``) or the tcgen05 GEMM."""
    global _LIBRARY_GEMM
    _LIBRARY_GEMM = bool(on)


def library_gemm() -> bool:
    return _LIBRARY_GEMM


def _lib(x: torch.Tensor, w) -> bool:
    return _LIBRARY_GEMM and x.is_cuda and isinstance(w, torch.Tensor)


# Activations of decode-size block-FP8 projections: "fp8" quantizes them per token and 128-wide k
# block (W8A8, per-k-block promotion on the tensor cores: the weight stream needs no widening),
# "bf16" keeps them exact (W8A16: the weight tiles are widened to bf16 in shared memory).
_FP8_BLOCK_ACT = "fp8"


def set_fp8_block_activations(mode: str) -> None:
    global _FP8_BLOCK_ACT
    if mode not in ("fp8", "bf16"):
        raise ValueError(f"fp8 block activations must be 'fp8' or 'bf16', got {mode!r}")
    _FP8_BLOCK_ACT = mode


def fp8_block_activations() -> str:
    return _FP8_BLOCK_ACT


def _w8a8_prefill(M: int, N: int, K: int, w) -> bool:
    """Prefill-size block-FP8 projection on the W8A8 promotion kernel (fp8 activation mode,
    128-aligned K and weight rows)."""
    return (_FP8_BLOCK_ACT == "fp8" and M > SKINNY_MAX and K % 128 == 0 and N % 128 == 0
            and w.scales.shape[1] >= K // 128)


def quantize_fp8_blocks(x: torch.Tensor, out: torch.Tensor | None = None,
                        scales: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token, per-128-column e4m3 quantization: ``s = max|x_block| / 448`` (1 for an
    all-zero block), ``q = satfinite(x / s)``.  Returns ``(q [M, K], s [M, K / 128])``."""
    M, K = x.shape
    assert K % 128 == 0
    if out is None:
        out = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    if scales is None:
        scales = torch.empty((M, K // 128), dtype=torch.float32, device=x.device)
    if x.is_cuda and x.dtype == torch.bfloat16 and x.stride(1) == 1:
        ext().quant_fp8_block(x, out, scales)
        return out, scales
    xb = x.float().view(M, K // 128, 128)
    s = xb.abs().amax(-1)
    s = torch.where(s > 0, s / FP8_MAX, torch.ones_like(s))
    out.copy_((xb / s[..., None]).clamp(-FP8_MAX, FP8_MAX).view(M, K).to(torch.float8_e4m3fn))
    scales.copy_(s)
    return out, scales


def dequantize_fp8_blocks(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    M, K = q.shape
    return (q.float().view(M, K // 128, 128) * s[..., None]).view(M, K)

_NUM_SMS: dict[int, int] = {}


def num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _NUM_SMS:
        _NUM_SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _NUM_SMS[idx]


def _pick_bn_wide(m: int, n: int, sms: int) -> int:
    """Pick the N tile (128 or 256) that minimises waves * tile-time for a wide GEMM."""
    best, best_cost = 256, float("inf")
    mb = math.ceil(m / 128)
    for bn, cost_per_tile in ((256, 2.0), (128, 1.08)):
        tiles = mb * math.ceil(n / bn)
        waves = math.ceil(tiles / sms)
        cost = waves * cost_per_tile
        if cost < best_cost - 1e-9:
            best, best_cost = bn, cost
    return best


def skinny_bn(m: int) -> int:
    for bn in (16, 32, 64, 128):
        if m <= bn:
            return bn
    raise ValueError(m)


def pick_splits(n_rows: int, k: int, sms: int, k_block: int = 64) -> int:
    """Split-K factor so that (row tiles x splits) covers the SMs, keeping >= 4 K-blocks."""
    tiles = math.ceil(n_rows / 128)
    kb = math.ceil(k / k_block)
    if tiles >= sms:
        return 1
    s = max(1, min(sms // tiles, kb // 4))
    return s


def _mx8_ref(x: torch.Tensor, w: "MXFP8Weight") -> torch.Tensor:
    """fp32 oracle of the MXFP8 GEMM: MXFP8-rounded activations times the MXFP8 weight."""
    xq, xs = quantize_mx8(x)
    return dequantize_mx8(xq, xs) @ w.dequant().t()


def _mx8_bf16(x: torch.Tensor, w: "MXFP8Weight", out: torch.Tensor) -> torch.Tensor:
    """bf16 ``out = x @ w^T`` on the block-scaled tensor cores: swapped operands and a
    transposed store for decode batches (<= 64 tokens), tokens as the 128-row operand above."""
    M = x.shape[0]
    if not x.is_cuda:
        out.copy_(_mx8_ref(x, w).to(out.dtype))
        return out
    xq, sf = mx8_quantize_device(x)
    if M <= 64:
        ext().gemm_mx8(w.q, xq, out, EPI_BF16_T, skinny_bn(M), 1, w.sf, sf)
    else:
        ext().gemm_mx8(xq, w.q, out, EPI_BF16, 128, 1, sf, w.sf)
    return out


def gemm_out(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
             bn: int | None = None) -> torch.Tensor:
    """``out[M, N] = x[M, K] @ w[N, K]^T`` in bf16 (wide regime, no split-K)."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16 if x.is_cuda else x.dtype, device=x.device)
    if isinstance(w, MXFP8Weight):
        return _mx8_bf16(x, w, out)
    if isinstance(w, FP8Weight):
        xq = quantize_fp8(x, w.in_scale)
        if not x.is_cuda:
            out.copy_(_fp8_ref(xq, w).to(out.dtype))
            return out
        ext().gemm_fp8(xq, w.q, out, EPI_BF16, bn or _pick_bn_wide(M, N, num_sms(x.device)), 1,
                       w.in_scale * w.w_scale)
        return out
    if isinstance(w, BlockFP8Weight):
        if not x.is_cuda:
            out.copy_((x.float() @ w.dequant_bf16_ref().float().t()).to(out.dtype))
            return out
        if _w8a8_prefill(M, N, K, w):
            xq, xs = quantize_fp8_blocks(x)
            ext().gemm_fp8_block_prefill(xq, w.q, out, w.scales, xs)
            return out
        ext().gemm_w8(x, w.q, out, EPI_BF16, bn or _pick_bn_wide(M, N, num_sms(x.device)), 1,
                      w.scales, 2, None, None)
        return out
    if not x.is_cuda:
        out.copy_((x.float() @ w.float().t()).to(out.dtype))
        return out
    if _lib(x, w):
        torch.mm(x, w.t(), out=out)
        return out
    if bn is None:
        bn = _pick_bn_wide(M, N, num_sms(x.device))
    ext().gemm(x, w, out, EPI_BF16, bn, 1, 0, 0)
    return out


def gemm_skinny_bf16(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Decode regime without split-K: swapped operands, transposed bf16 store."""
    M, K = x.shape
    N = w.shape[0]
    if isinstance(w, (FP8Weight, MXFP8Weight)):  # row-major regime (no transposed FP8 store)
        return gemm_out(x, w, out)
    if isinstance(w, BlockFP8Weight):
        if out is None:
            out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
        if not x.is_cuda:
            return gemm_out(x, w, out)
        ext().gemm_w8(w.q, x, out, EPI_BF16_T, skinny_bn(M), 1, w.scales, 1, None, None)
        return out
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    if not x.is_cuda:
        out.copy_((x.float() @ w.float().t()).to(out.dtype))
        return out
    if _lib(x, w):
        torch.mm(x, w.t(), out=out)
        return out
    ext().gemm(w, x, out, EPI_BF16_T, skinny_bn(M), 1, 0, 0)
    return out


def gemm_accumulate(x: torch.Tensor, w: torch.Tensor, acc: torch.Tensor,
                    splits: int | None = None) -> torch.Tensor:
    """``acc[M, N] += x @ w^T`` in fp32 (split-K; the consumer clears ``acc`` after use).

    ``acc`` must be zero on entry (the fused consumers leave it zeroed).
    """
    M, K = x.shape
    N = w.shape[0]
    assert acc.dtype == torch.float32 and acc.shape[0] >= M and acc.shape[1] == N
    if isinstance(w, MXFP8Weight):
        if not x.is_cuda:
            acc[:M].add_(_mx8_ref(x, w))
            return acc
        xq, sf = mx8_quantize_device(x)
        sms = num_sms(x.device)
        if M <= SKINNY_MAX:
            tiles = math.ceil(N / 128)
            s = splits if splits is not None else (pick_splits(N, K, sms, 128) if tiles < sms else -1)
            ext().gemm_mx8(w.q, xq, acc, EPI_F32_RED_T, skinny_bn(M), s, w.sf, sf)
        else:
            rows = math.ceil(M / 128) * 128 * math.ceil(N / 128)
            s = splits if splits is not None else pick_splits(rows, K, sms, 128)
            ext().gemm_mx8(xq, w.q, acc, EPI_F32_RED, 128, s, sf, w.sf)
        return acc
    if isinstance(w, FP8Weight):
        xq = quantize_fp8(x, w.in_scale)
        if not x.is_cuda:
            acc[:M].add_(_fp8_ref(xq, w))
            return acc
        sms = num_sms(x.device)
        if M <= SKINNY_MAX:
            s = splits if splits is not None else pick_splits(N, K, sms, 128)
            ext().gemm_fp8(w.q, xq, acc, EPI_F32_RED_T, skinny_bn(M), s, w.in_scale * w.w_scale)
        else:
            rows = math.ceil(M / 128) * 128 * math.ceil(N / 128)
            s = splits if splits is not None else pick_splits(rows, K, sms, 128)
            ext().gemm_fp8(xq, w.q, acc, EPI_F32_RED, 128, s, w.in_scale * w.w_scale)
        return acc
    if isinstance(w, BlockFP8Weight):
        if not x.is_cuda:
            acc[:M].add_(x.float() @ w.dequant_bf16_ref().float().t())
            return acc
        sms = num_sms(x.device)
        if (M <= 32 and _FP8_BLOCK_ACT == "fp8" and K % 128 == 0 and N % 128 == 0 and not splits
                and w.scales.shape[1] >= K // 128):
            # W8A8: e4m3 weights and per-block e4m3 activations straight into the tensor cores
            # (measured faster up to 32 tokens; at 64 the 64-column promotion epilogue is the
            # limit and the W8A16 converter path wins on most shapes)
            xq, xs = quantize_fp8_blocks(x)
            tiles = math.ceil(N / 128)
            s = pick_splits(N, K, sms, 128) if tiles < sms else -1
            ext().gemm_fp8_block(w.q, xq, acc, skinny_bn(M), s, w.scales, xs)
        elif M <= SKINNY_MAX:
            s = splits if splits is not None else pick_splits(N, K, sms)
            ext().gemm_w8(w.q, x, acc, EPI_F32_RED_T, skinny_bn(M), s, w.scales, 1, None, None)
        else:
            rows = math.ceil(M / 128) * 128 * math.ceil(N / 128)
            s = splits if splits is not None else pick_splits(rows, K, sms)
            ext().gemm_w8(x, w.q, acc, EPI_F32_RED, 128, s, w.scales, 2, None, None)
        return acc
    if not x.is_cuda:
        acc[:M].add_(x.float() @ w.float().t())
        return acc
    if _lib(x, w):
        # acc is zero on entry: one cuBLAS call with an fp32 output (bf16 inputs)
        torch.mm(x, w.t(), out_dtype=torch.float32, out=acc[:M])
        return acc
    # splits=None: split-K when the row tiles alone under-fill the SMs (measured faster for
    # the small qkv / o projections), stream-K (-1: every persistent CTA takes an equal share
    # of (tile, k-block) units) when there are more tiles than SMs.
    if splits is None:
        rows = N if M <= SKINNY_MAX else math.ceil(M / 128) * 128 * math.ceil(N / 128)
        tiles = math.ceil(rows / 128)
        s = pick_splits(rows, K, num_sms(x.device)) if tiles < num_sms(x.device) else -1
    else:
        s = splits
    if M <= SKINNY_MAX:
        ext().gemm(w, x, acc, EPI_F32_RED_T, skinny_bn(M), s, 0, 0)
    else:
        ext().gemm(x, w, acc, EPI_F32_RED, 128, s, 0, 0)
    return acc


def gemm_silu(x: torch.Tensor, w_gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused ``silu(x @ g^T) * (x @ u^T)`` where ``w_gu`` interleaves gate/up rows in blocks of
    ``SILU_BLOCK`` (see :func:`interleave_gate_up`)."""
    M, K = x.shape
    N2 = w_gu.shape[0]
    if out is None:
        out = torch.empty((M, N2 // 2), dtype=torch.bfloat16, device=x.device)
    if isinstance(w_gu, MXFP8Weight):
        if not x.is_cuda:
            out.copy_(silu_mul_ref(_mx8_ref(x, w_gu), SILU_BLOCK).to(out.dtype))
            return out
        from .activation import silu_mul

        gu = _mx8_bf16(x, w_gu, torch.empty((M, N2), dtype=torch.bfloat16, device=x.device))
        return silu_mul(gu, out=out, blk=SILU_BLOCK)
    if isinstance(w_gu, FP8Weight):
        xq = quantize_fp8(x, w_gu.in_scale)
        if not x.is_cuda:
            out.copy_(silu_mul_ref(_fp8_ref(xq, w_gu), SILU_BLOCK).to(out.dtype))
            return out
        ext().gemm_fp8(xq, w_gu.q, out, EPI_SILU_BF16, 2 * SILU_BLOCK, 1, w_gu.in_scale * w_gu.w_scale)
        return out
    if isinstance(w_gu, BlockFP8Weight):
        if not x.is_cuda:
            y = x.float() @ w_gu.dequant_bf16_ref().float().t()
            out.copy_(silu_mul_ref(y, SILU_BLOCK).to(out.dtype))
            return out
        if _w8a8_prefill(M, N2, K, w_gu):
            from .activation import silu_mul

            xq, xs = quantize_fp8_blocks(x)
            gu = torch.empty((M, N2), dtype=torch.bfloat16, device=x.device)
            ext().gemm_fp8_block_prefill(xq, w_gu.q, gu, w_gu.scales, xs)
            return silu_mul(gu, out=out, blk=SILU_BLOCK)
        ext().gemm_w8(x, w_gu.q, out, EPI_SILU_BF16, 2 * SILU_BLOCK, 1, w_gu.scales, 2, None, None)
        return out
    if not x.is_cuda:
        y = x.float() @ w_gu.float().t()
        out.copy_(silu_mul_ref(y, SILU_BLOCK).to(out.dtype))
        return out
    if _lib(x, w_gu):
        from .activation import silu_mul

        return silu_mul(torch.mm(x, w_gu.t()), out=out, blk=SILU_BLOCK)
    ext().gemm(x, w_gu, out, EPI_SILU_BF16, 2 * SILU_BLOCK, 1, 0, 0)
    return out


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, blk: int = SILU_BLOCK) -> torch.Tensor:
    """Rows ``[g[0:blk], u[0:blk], g[blk:2blk], u[blk:2blk], ...]`` (requires I % blk == 0)."""
    I, K = gate.shape
    assert up.shape == gate.shape and I % blk == 0
    return torch.stack([gate.view(I // blk, blk, K), up.view(I // blk, blk, K)], dim=1).reshape(2 * I, K)


def silu_mul_ref(y: torch.Tensor, blk: int) -> torch.Tensor:
    """fp32 reference of SwiGLU on a [T, 2I] tensor whose gate/up columns are interleaved in
    blocks of ``blk`` (``blk == 0``: first half gate, second half up)."""
    T, I2 = y.shape
    I = I2 // 2
    if blk > 0:
        v = y.view(T, I // blk, 2, blk)
        g, u = v[:, :, 0, :].reshape(T, I), v[:, :, 1, :].reshape(T, I)
    else:
        g, u = y[:, :I], y[:, I:]
    g = g.float()
    return torch.nn.functional.silu(g) * u.float()
