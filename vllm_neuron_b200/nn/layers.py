"""Column/row-parallel linears and sharded embeddings (see the package docstring).

Sharding conventions (as in the reference and in vLLM):

* ``ColumnParallelLinear``: ``W [out, in]`` split along ``out``; each rank produces its slice of
  the output features (optionally all-gathered back to the full width).
* ``RowParallelLinear``: ``W [out, in]`` split along ``in``; each rank multiplies its slice of the
  input features and the partial sums are all-reduced (or reduce-scattered over tokens under
  sequence parallelism).  A bias is added once, after the reduction.
* ``VocabParallelEmbedding``: table rows split by vocabulary range; out-of-range ids give zero
  rows, so the sum over ranks is the full embedding.
* ``EmbedDimShardedEmbedding``: table columns split; the hidden slices are all-gathered.
"""
from __future__ import annotations

import torch

from .. import ops
from ..ops import linear as L
from ..parallel.comm import SINGLE, GroupComm


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """``[start, end)`` of ``rank``'s equal shard of ``total`` (must divide evenly)."""
    if total % world:
        raise ValueError(f"{total} does not split evenly over {world} ranks")
    n = total // world
    return rank * n, (rank + 1) * n


def _matmul(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x [T, K] @ w[N, K]^T`` on the tcgen05 GEMM (skinny kernel for decode-sized T)."""
    if x.is_cuda and x.dtype == torch.bfloat16:
        if x.shape[0] <= L.SKINNY_MAX:
            return L.gemm_skinny_bf16(x, w, out=out)
        return L.gemm_out(x, w, out=out)
    y = x.float() @ w.float().t()
    if out is not None:
        out.copy_(y.to(out.dtype))
        return out
    return y.to(x.dtype)


class _Linear(torch.nn.Module):
    def __init__(self, weight_shape: tuple[int, int], bias_size: int | None, comm: GroupComm,
                 device, dtype):
        super().__init__()
        self.comm = comm
        self.weight = torch.nn.Parameter(torch.empty(weight_shape, device=device, dtype=dtype),
                                         requires_grad=False)
        self.bias = (torch.nn.Parameter(torch.zeros(bias_size, device=device, dtype=dtype), requires_grad=False)
                     if bias_size is not None else None)

    def reset_parameters(self, std: float = 0.02, generator: torch.Generator | None = None):
        with torch.no_grad():
            self.weight.normal_(0.0, std, generator=generator)
            if self.bias is not None:
                self.bias.zero_()


class ColumnParallelLinear(_Linear):
    """``y[:, shard] = x @ W[shard]^T (+ b[shard])``; ``gather_output`` all-gathers the full
    width (reference: ColumnParallelLinear, nn/cpl.py:27-143)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 comm: GroupComm = SINGLE, gather_output: bool = False, device=None,
                 dtype=torch.bfloat16):
        self.in_features, self.out_features = in_features, out_features
        self.start, self.end = shard_range(out_features, comm.world, comm.rank)
        super().__init__((self.end - self.start, in_features), self.end - self.start if bias else None,
                         comm, device, dtype)
        self.gather_output = gather_output

    def load_full_weight(self, w: torch.Tensor, b: torch.Tensor | None = None):
        """Copy this rank's rows out of the unsharded ``w [out, in]`` (and ``b [out]``)."""
        with torch.no_grad():
            self.weight.copy_(w[self.start:self.end])
            if b is not None and self.bias is not None:
                self.bias.copy_(b[self.start:self.end])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = _matmul(x, self.weight)
        if self.bias is not None:
            y = y + self.bias
        if self.gather_output and self.comm.world > 1:
            y = self.comm.all_gather(y, dim=-1)
        return y


class MergedColumnParallelLinear(ColumnParallelLinear):
    """Several column-parallel outputs in one GEMM (e.g. gate and up): each part is sharded
    separately and the shards are concatenated, so rank r holds ``[gate_r | up_r]``."""

    def __init__(self, in_features: int, out_sizes: list[int], bias: bool = False,
                 comm: GroupComm = SINGLE, device=None, dtype=torch.bfloat16):
        self.out_sizes = list(out_sizes)
        for n in out_sizes:
            shard_range(n, comm.world, comm.rank)
        torch.nn.Module.__init__(self)
        self.in_features, self.out_features = in_features, sum(out_sizes)
        self.start, self.end = 0, sum(out_sizes) // comm.world
        _Linear.__init__(self, (self.end, in_features), self.end if bias else None, comm, device, dtype)
        self.gather_output = False

    def load_full_weight(self, w: torch.Tensor, b: torch.Tensor | None = None):
        parts_w, parts_b, off = [], [], 0
        for n in self.out_sizes:
            s, e = shard_range(n, self.comm.world, self.comm.rank)
            parts_w.append(w[off + s:off + e])
            if b is not None:
                parts_b.append(b[off + s:off + e])
            off += n
        with torch.no_grad():
            self.weight.copy_(torch.cat(parts_w, 0))
            if b is not None and self.bias is not None:
                self.bias.copy_(torch.cat(parts_b, 0))


class QKVParallelLinear(MergedColumnParallelLinear):
    """Fused q|k|v projection with heads split over ranks.  When the KV heads are fewer than
    the ranks, each KV head is replicated on ``world / num_kv_heads`` ranks (reference:
    fused_qkv_weight_loader, utils/weight_loader.py)."""

    def __init__(self, hidden: int, head_dim: int, num_heads: int, num_kv_heads: int,
                 bias: bool = False, comm: GroupComm = SINGLE, device=None, dtype=torch.bfloat16):
        W = comm.world
        if num_heads % W:
            raise ValueError("query heads must split evenly over the TP ranks")
        self.kv_rep = max(1, W // num_kv_heads)
        self.kv_local = max(1, num_kv_heads // W)
        self.head_dim, self.num_heads, self.num_kv_heads = head_dim, num_heads, num_kv_heads
        q_local = num_heads // W * head_dim
        kv_local = self.kv_local * head_dim
        torch.nn.Module.__init__(self)
        self.in_features = hidden
        self.out_sizes = [num_heads * head_dim, num_kv_heads * head_dim, num_kv_heads * head_dim]
        self.out_features = q_local + 2 * kv_local
        self.start, self.end = 0, self.out_features
        _Linear.__init__(self, (self.out_features, hidden), self.out_features if bias else None,
                         comm, device, dtype)
        self.gather_output = False

    def load_full_weight(self, w: torch.Tensor, b: torch.Tensor | None = None):
        D, W, r = self.head_dim, self.comm.world, self.comm.rank
        nq = self.num_heads * D
        nkv = self.num_kv_heads * D
        q = w[:nq].view(self.num_heads, D, -1)
        k = w[nq:nq + nkv].view(self.num_kv_heads, D, -1)
        v = w[nq + nkv:].view(self.num_kv_heads, D, -1)
        qh = self.num_heads // W
        kv0 = (r // self.kv_rep) * self.kv_local
        parts = [q[r * qh:(r + 1) * qh], k[kv0:kv0 + self.kv_local], v[kv0:kv0 + self.kv_local]]
        with torch.no_grad():
            self.weight.copy_(torch.cat([p.reshape(-1, w.shape[1]) for p in parts], 0))
            if b is not None and self.bias is not None:
                bq, bk, bv = b[:nq].view(-1, D), b[nq:nq + nkv].view(-1, D), b[nq + nkv:].view(-1, D)
                self.bias.copy_(torch.cat([bq[r * qh:(r + 1) * qh].reshape(-1),
                                           bk[kv0:kv0 + self.kv_local].reshape(-1),
                                           bv[kv0:kv0 + self.kv_local].reshape(-1)]))


class RowParallelLinear(_Linear):
    """``y = sum_ranks x[:, shard] @ W[:, shard]^T (+ b)``; ``reduce="all"`` all-reduces,
    ``reduce="scatter"`` reduce-scatters over tokens (sequence parallelism), ``reduce=None``
    leaves the partial sum (the caller fuses the reduction, e.g. with residual + RMSNorm)
    (reference: RowParallelLinear, nn/rpl.py:23-154)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 comm: GroupComm = SINGLE, reduce: str | None = "all", input_is_parallel: bool = True,
                 device=None, dtype=torch.bfloat16):
        self.in_features, self.out_features = in_features, out_features
        self.start, self.end = shard_range(in_features, comm.world, comm.rank)
        super().__init__((out_features, self.end - self.start), out_features if bias else None, comm,
                         device, dtype)
        if reduce not in ("all", "scatter", None):
            raise ValueError("reduce must be 'all', 'scatter' or None")
        self.reduce = reduce
        self.input_is_parallel = input_is_parallel

    def load_full_weight(self, w: torch.Tensor, b: torch.Tensor | None = None):
        with torch.no_grad():
            self.weight.copy_(w[:, self.start:self.end])
            if b is not None and self.bias is not None:
                self.bias.copy_(b)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.input_is_parallel:
            x = x[..., self.start:self.end].contiguous()
        y = _matmul(x, self.weight)
        if self.comm.world > 1:
            if self.reduce == "all":
                self.comm.all_reduce_(y)
            elif self.reduce == "scatter":
                y = self.comm.reduce_scatter(y)
        if self.bias is not None and self.reduce is not None:
            y = y + self.bias
        return y


class VocabParallelEmbedding(torch.nn.Module):
    """Vocabulary-sharded lookup (csrc ``embedding_kernel``); ``reduce="all"`` all-reduces the
    rows, ``"scatter"`` reduce-scatters them over tokens (enters sequence parallelism)
    (reference: VocabDimShardedEmbedding, nn/embedding.py:23-249)."""

    def __init__(self, num_embeddings: int, embedding_dim: int, comm: GroupComm = SINGLE,
                 reduce: str | None = "all", device=None, dtype=torch.bfloat16):
        super().__init__()
        self.comm = comm
        self.num_embeddings, self.embedding_dim = num_embeddings, embedding_dim
        per = -(-num_embeddings // comm.world)
        self.vocab_start = comm.rank * per
        self.vocab_end = min(num_embeddings, self.vocab_start + per)
        self.weight = torch.nn.Parameter(torch.zeros(per, embedding_dim, device=device, dtype=dtype),
                                         requires_grad=False)
        self.reduce = reduce

    def load_full_weight(self, table: torch.Tensor):
        with torch.no_grad():
            n = self.vocab_end - self.vocab_start
            self.weight[:n].copy_(table[self.vocab_start:self.vocab_end])

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        y = ops.embedding(ids.to(torch.int32), self.weight, self.vocab_start, self.vocab_end)
        if self.comm.world > 1:
            if self.reduce == "all":
                self.comm.all_reduce_(y)
            elif self.reduce == "scatter":
                y = self.comm.reduce_scatter(y)
        return y


class EmbedDimShardedEmbedding(torch.nn.Module):
    """Hidden-dimension-sharded lookup followed by an all-gather of the slices (reference:
    EmbedDimShardedEmbedding, nn/embedding.py:252-433)."""

    def __init__(self, num_embeddings: int, embedding_dim: int, comm: GroupComm = SINGLE,
                 device=None, dtype=torch.bfloat16):
        super().__init__()
        self.comm = comm
        self.start, self.end = shard_range(embedding_dim, comm.world, comm.rank)
        self.weight = torch.nn.Parameter(torch.zeros(num_embeddings, self.end - self.start, device=device,
                                                     dtype=dtype), requires_grad=False)

    def load_full_weight(self, table: torch.Tensor):
        with torch.no_grad():
            self.weight.copy_(table[:, self.start:self.end])

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        y = ops.embedding(ids.to(torch.int32), self.weight)
        if self.comm.world > 1:
            y = self.comm.all_gather(y, dim=-1)
        return y
