"""Block packing of variable-size images for the vision encoder.

The vision encoder attends only inside an image (inside a frame for videos), so the patches of
several images can share one fixed-size block of ``block_size`` rows as long as each query row
only sees the keys of its own image.  Packing turns the per-image encoder loop into a few
equal-shape blocks:

* every projection / MLP GEMM of the encoder runs once over ``num_blocks * block_size`` rows,
* attention runs as one batched call over the blocks with per-row key bounds ``[lo, hi)``,
* the shapes depend only on ``num_blocks`` (chosen from a short bucket list), so the whole
  encoder forward can be captured in one CUDA graph per bucket and replayed for any mix of
  images that fits.

Plan construction is host-side integer work on the image sizes; the layout moves (scatter into
blocks, gather of the merged rows back into image order) are single index ops on the device.

Reference behaviour: vllm_neuron/model/qwen3_vl/utils/vision_block_packing.py (first-fit
decreasing assignment, the one-item-per-block mode with group ids, block-local attention bounds
per frame, post-merger unpack indices, bucket selection padded to the vision-DP degree).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class PackPlan:
    """Where each item (image or frame group) sits in the packed layout.

    ``bins[b]`` lists the items of block ``b`` in ascending item order (their order inside the
    block); ``block_of[i]`` / ``offset_of[i]`` give item ``i``'s block and first row in it.
    """

    bins: list[list[int]]
    block_size: int
    sizes: list[int]
    block_of: list[int]
    offset_of: list[int]

    @property
    def num_blocks(self) -> int:
        return len(self.bins)

    @property
    def rows(self) -> int:
        return self.num_blocks * self.block_size

    def used(self, b: int) -> int:
        return sum(self.sizes[i] for i in self.bins[b])

    def fill(self) -> float:
        """Fraction of packed rows that hold real tokens."""
        return sum(self.sizes) / max(1, self.rows)


def _finish(bins: list[list[int]], block_size: int, sizes: list[int]) -> PackPlan:
    block_of = [-1] * len(sizes)
    offset_of = [0] * len(sizes)
    for b, items in enumerate(bins):
        items.sort()
        off = 0
        for i in items:
            block_of[i], offset_of[i] = b, off
            off += sizes[i]
    return PackPlan(bins, block_size, list(sizes), block_of, offset_of)


def pack_items(sizes: list[int], block_size: int, num_blocks: int | None = None,
               one_item_per_block: bool = False, group_ids: list[int] | None = None) -> PackPlan:
    """Assign items of ``sizes`` tokens to blocks of ``block_size`` rows.

    Default: first-fit decreasing (largest item first, each into the first block with room).
    ``one_item_per_block``: blocks are taken in item order and never shared between groups;
    consecutive items with the same ``group_ids`` entry (a video's frames) fill a block before
    the next one is opened, so a cached item can be addressed by its block range.

    ``num_blocks`` fixes the block count (unused blocks stay empty, e.g. to reach a bucket);
    ``None`` opens as many as needed.  Raises ``ValueError`` when an item is larger than a block
    or the items do not fit.
    """
    for i, s in enumerate(sizes):
        if s <= 0:
            raise ValueError(f"item {i} has {s} tokens")
        if s > block_size:
            raise ValueError(f"item {i} has {s} tokens, more than the block size {block_size}; "
                             "an image's attention has to stay inside one block")
    limit = math.inf if num_blocks is None else num_blocks
    bins: list[list[int]] = []
    if one_item_per_block:
        gid = list(range(len(sizes))) if group_ids is None else list(group_ids)
        if len(gid) != len(sizes):
            raise ValueError("group_ids must have one entry per item")
        room, prev = 0, object()
        for i, s in enumerate(sizes):
            if gid[i] != prev or room < s:
                if len(bins) + 1 > limit:
                    raise ValueError(f"item {i} ({s} tokens) does not fit in {num_blocks} blocks "
                                     f"of {block_size}")
                bins.append([])
                room, prev = block_size, gid[i]
            bins[-1].append(i)
            room -= s
    else:
        if group_ids is not None:
            raise ValueError("group_ids only applies with one_item_per_block")
        room: list[int] = []
        for i in sorted(range(len(sizes)), key=lambda j: (-sizes[j], j)):
            s = sizes[i]
            for b, r in enumerate(room):
                if r >= s:
                    bins[b].append(i)
                    room[b] -= s
                    break
            else:
                if len(bins) + 1 > limit:
                    raise ValueError(f"item {i} ({s} tokens) does not fit in {num_blocks} blocks "
                                     f"of {block_size}")
                bins.append([i])
                room.append(block_size - s)
    if num_blocks is not None:
        bins += [[] for _ in range(num_blocks - len(bins))]
    return _finish(bins, block_size, sizes)


def select_bucket(total_tokens: int, buckets: list[int], block_size: int, dp: int = 1) -> tuple[int, int]:
    """Smallest bucket holding ``total_tokens`` and its block count, padded to a multiple of the
    vision-DP degree ``dp`` so every replica encodes the same number of blocks."""
    if not buckets:
        raise ValueError("num_vision_tokens_buckets is empty")
    for bucket in sorted(buckets):
        if bucket >= total_tokens:
            nb = -(-bucket // block_size)
            return bucket, -(-nb // dp) * dp
    raise ValueError(f"{total_tokens} vision tokens exceed the largest bucket {max(buckets)}")


def plan_for_buckets(sizes: list[int], block_size: int, buckets: list[int] | None,
                     dp: int = 1) -> PackPlan:
    """First-fit-decreasing plan whose block count comes from ``buckets`` (the smallest bucket
    whose blocks hold the items; a larger one when fragmentation needs more blocks).  Without
    buckets the block count is the packed minimum rounded up to ``dp``."""
    if not buckets:
        plan = pack_items(sizes, block_size)
        nb = -(-max(1, plan.num_blocks) // dp) * dp
        return pack_items(sizes, block_size, nb)
    total = sum(sizes)
    for bucket in sorted(b for b in buckets if b >= total):
        _, nb = select_bucket(bucket, [bucket], block_size, dp)
        try:
            return pack_items(sizes, block_size, nb)
        except ValueError:
            continue
    raise ValueError(f"images of {sizes} tokens do not pack into any bucket of {sorted(buckets)} "
                     f"with blocks of {block_size}")


def scatter_index(plan: PackPlan) -> torch.Tensor:
    """``dst[t]`` = packed row of flat token ``t`` (items concatenated in item order)."""
    parts = [torch.arange(n) + plan.block_of[i] * plan.block_size + plan.offset_of[i]
             for i, n in enumerate(plan.sizes)]
    return torch.cat(parts) if parts else torch.zeros(0, dtype=torch.long)


def to_blocks(flat: torch.Tensor, plan: PackPlan, dst: torch.Tensor | None = None) -> torch.Tensor:
    """``flat [tokens, ...]`` -> ``[num_blocks * block_size, ...]`` with zero padding rows."""
    dst = scatter_index(plan) if dst is None else dst
    out = flat.new_zeros((plan.rows,) + tuple(flat.shape[1:]))
    out.index_copy_(0, dst.to(flat.device), flat)
    return out


def block_bounds(plan: PackPlan, frames: list[int] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per packed row, the block-local key range ``[lo, hi)`` it attends to.

    Item ``i`` is split into ``frames[i]`` equal frames (default 1) that attend separately.
    Padding rows attend to themselves only (a one-key range keeps the softmax finite; their
    outputs are never read)."""
    bs = plan.block_size
    ar = torch.arange(bs, dtype=torch.int32)
    lo = ar.repeat(plan.num_blocks).view(plan.num_blocks, bs).clone()
    hi = lo + 1
    for i, n in enumerate(plan.sizes):
        f = 1 if frames is None else frames[i]
        if n % f:
            raise ValueError(f"item {i}: {n} tokens do not split into {f} frames")
        per = n // f
        b, o = plan.block_of[i], plan.offset_of[i]
        for k in range(f):
            s = o + k * per
            lo[b, s:s + per] = s
            hi[b, s:s + per] = s + per
    return lo, hi


def bounds_mask(lo: torch.Tensor, hi: torch.Tensor) -> torch.Tensor:
    """Boolean attention mask ``[num_blocks, 1, bs, bs]`` from per-row bounds (True = visible)."""
    j = torch.arange(lo.shape[1], device=lo.device, dtype=lo.dtype)
    return ((j[None, None, :] >= lo[:, :, None]) & (j[None, None, :] < hi[:, :, None])).unsqueeze(1)


def unpack_index(plan: PackPlan, merge: int) -> torch.Tensor:
    """Gather index restoring item order after the ``merge``-row spatial merger: entry ``r`` is
    the merged packed row of the ``r``-th merged output row (items in item order)."""
    if plan.block_size % merge:
        raise ValueError(f"block size {plan.block_size} is not a multiple of the merge group {merge}")
    mb = plan.block_size // merge
    parts = []
    for i, n in enumerate(plan.sizes):
        if n % merge:
            raise ValueError(f"item {i}: {n} tokens are not a multiple of the merge group {merge}")
        parts.append(torch.arange(n // merge) + plan.block_of[i] * mb + plan.offset_of[i] // merge)
    return torch.cat(parts) if parts else torch.zeros(0, dtype=torch.long)
