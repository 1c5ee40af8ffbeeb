"""Vision block packing: the plan (first-fit decreasing, one item per block with groups, bucket
selection padded to the vision-DP degree), the layout moves, the per-frame attention bounds,
and the packed Qwen3-VL encoder against the per-image encoder (fp32, CPU)."""
import pytest
import torch

from vllm_neuron_b200.config import VisionConfig
from vllm_neuron_b200.models import vision_packing as VP


def _check_plan(plan, sizes):
    seen = sorted(i for b in plan.bins for i in b)
    assert seen == list(range(len(sizes)))
    for b in range(plan.num_blocks):
        assert plan.used(b) <= plan.block_size
        off = 0
        for i in plan.bins[b]:  # ascending item order, contiguous offsets
            assert plan.block_of[i] == b and plan.offset_of[i] == off
            off += sizes[i]


def test_ffd_packs_largest_first():
    sizes = [300, 700, 200, 500, 400, 100]
    plan = VP.pack_items(sizes, 1000)
    _check_plan(plan, sizes)
    # FFD: 700 + 300, then 500 + 400 + 100, then 200
    assert [sorted(b) for b in plan.bins] == [[0, 1], [3, 4, 5], [2]]
    assert plan.fill() == pytest.approx(2200 / 3000)
    with pytest.raises(ValueError):
        VP.pack_items([1200], 1000)
    with pytest.raises(ValueError):
        VP.pack_items(sizes, 1000, num_blocks=2)
    padded = VP.pack_items(sizes, 1000, num_blocks=5)
    assert padded.num_blocks == 5 and padded.bins[3] == [] and padded.bins[4] == []


def test_one_item_per_block_groups_share_only_their_own_blocks():
    sizes = [100, 100, 100, 200, 50]
    plan = VP.pack_items(sizes, 250, one_item_per_block=True, group_ids=[0, 0, 0, 1, 2])
    _check_plan(plan, sizes)
    assert plan.bins == [[0, 1], [2], [3], [4]]
    plan = VP.pack_items(sizes, 250, one_item_per_block=True)
    assert plan.bins == [[0], [1], [2], [3], [4]]
    with pytest.raises(ValueError):
        VP.pack_items(sizes, 250, num_blocks=3, one_item_per_block=True)
    with pytest.raises(ValueError):
        VP.pack_items(sizes, 250, group_ids=[0] * 5)


def test_bucket_selection_and_dp_padding():
    assert VP.select_bucket(3000, [2048, 4096, 8192], 1024) == (4096, 4)
    assert VP.select_bucket(3000, [2048, 4096, 8192], 1024, dp=3) == (4096, 6)
    with pytest.raises(ValueError):
        VP.select_bucket(9000, [2048, 4096, 8192], 1024)
    # fragmentation: 3 x 600 tokens fit a 2048 bucket by count but need 3 blocks of 1024
    plan = VP.plan_for_buckets([600, 600, 600], 1024, [2048, 4096])
    assert plan.num_blocks == 4
    plan = VP.plan_for_buckets([600, 600, 600], 1024, None, dp=2)
    assert plan.num_blocks == 4


def test_layout_round_trip_bounds_and_unpack():
    sizes = [8, 16, 4, 12]
    plan = VP.pack_items(sizes, 20)
    _check_plan(plan, sizes)
    flat = torch.arange(sum(sizes), dtype=torch.float32)[:, None].repeat(1, 3)
    packed = VP.to_blocks(flat, plan)
    dst = VP.scatter_index(plan)
    assert torch.equal(packed[dst], flat)
    pad = torch.ones(plan.rows, dtype=torch.bool)
    pad[dst] = False
    assert torch.all(packed[pad] == 0)
    # item 1 (16 rows) as 2 frames of 8
    lo, hi = VP.block_bounds(plan, frames=[1, 2, 1, 1])
    b, o = plan.block_of[1], plan.offset_of[1]
    assert lo[b, o:o + 8].tolist() == [o] * 8 and hi[b, o:o + 8].tolist() == [o + 8] * 8
    assert lo[b, o + 8:o + 16].tolist() == [o + 8] * 8
    m = VP.bounds_mask(lo, hi)
    assert m.shape == (plan.num_blocks, 1, 20, 20)
    assert torch.all(m.sum(-1) >= 1)  # every row (padding too) sees at least one key
    # merged rows (groups of 4) return to item order
    merged = flat.view(-1, 4, 3)[:, 0, 0]            # first token of each merge group
    pm = packed.view(-1, 4, 3)[:, 0, 0]
    idx = VP.unpack_index(plan, 4)
    assert torch.equal(pm[idx], merged)


def _vision(seed=0, tp=None):
    from vllm_neuron_b200.models.qwen3_vl import Qwen3VLVision

    vc = dict(hidden_size=32, intermediate_size=64, num_heads=2, depth=3, patch_size=4,
              temporal_patch_size=2, spatial_merge_size=2, out_hidden_size=48,
              num_position_embeddings=16, deepstack_visual_indexes=[0, 2])
    v = Qwen3VLVision(vc, torch.device("cpu"), torch.float32)
    g = torch.Generator().manual_seed(seed)
    for p in v.parameters():
        p.data.copy_(torch.randn(p.shape, generator=g) * 0.1)
    return v


def test_packed_encoder_matches_per_image():
    v = _vision()
    grids = [(1, 4, 8), (2, 4, 4), (1, 8, 8), (1, 2, 2)]  # the second is a 2-frame video
    n = sum(t * h * w for t, h, w in grids)
    pix = torch.randn(n, 3 * 2 * 16, generator=torch.Generator().manual_seed(1))
    emb, deep = v(pix, grids)
    for bs in (64, 96):
        plan = VP.plan_for_buckets([t * h * w for t, h, w in grids], bs, None)
        pe, pd = v.forward_packed(pix, grids, plan)
        assert pe.shape == emb.shape and pd.shape == deep.shape
        assert torch.allclose(pe, emb, atol=1e-5, rtol=1e-4), (pe - emb).abs().max()
        assert torch.allclose(pd, deep, atol=1e-5, rtol=1e-4)


def test_video_frames_attend_separately():
    """Frames of one video do not attend to each other (the per-image path splits them too)."""
    v = _vision(3)
    grids = [(2, 4, 4)]
    pix = torch.randn(32, 96, generator=torch.Generator().manual_seed(2))
    e2, _ = v(pix, grids)
    e_a, _ = v(pix[:16], [(1, 4, 4)])
    e_b, _ = v(pix[16:], [(1, 4, 4)])
    # position embeddings and rotary are per frame position, so frame 2 alone equals its half
    assert torch.allclose(e2[:4], e_a, atol=1e-5) and torch.allclose(e2[4:], e_b, atol=1e-5)


def test_vision_config_keys():
    c = VisionConfig.from_dict({"vision_attention_block_size": 1024, "max_vision_seq_len": 5000})
    assert c.num_vision_tokens_buckets == [1024, 2048, 4096, 5120]
    assert c.resolve_tp_dp(8) == (1, 8)
    c = VisionConfig.from_dict({"tp_size": 2})
    assert c.resolve_tp_dp(8) == (2, 4)
    with pytest.raises(ValueError):
        VisionConfig.from_dict({"tp_size": 3}).resolve_tp_dp(8)
    with pytest.raises(ValueError):
        VisionConfig.from_dict({"vision_attention_block_size": 1022})
    with pytest.raises(ValueError):
        VisionConfig.from_dict({"no_such_key": 1})
    assert VisionConfig.from_additional_config({"neuron_config": {}}) is None


def test_mxfp8_vision_weights():
    """Qwen3-VL vision linears (input widths in 128s) as MXFP8 weights: the encoder runs them
    through the MXFP8 oracle on CPU and stays close to the bf16-weight encoder."""
    from vllm_neuron_b200.models.qwen3_vl import Qwen3VLVision
    from vllm_neuron_b200.ops import linear as L

    vc = dict(hidden_size=128, intermediate_size=256, num_heads=2, depth=2, patch_size=8,
              temporal_patch_size=2, spatial_merge_size=2, out_hidden_size=64,
              num_position_embeddings=16, deepstack_visual_indexes=[0])
    v = Qwen3VLVision(vc, torch.device("cpu"), torch.float32)
    g = torch.Generator().manual_seed(4)
    for p in v.parameters():
        p.data.copy_(torch.randn(p.shape, generator=g) * 0.05)
    grids = [(1, 4, 4), (1, 4, 8)]
    pix = torch.randn(48, 3 * 2 * 64, generator=g)
    ref, ref_d = v(pix, grids)

    from vllm_neuron_b200.models.qwen3_vl import quantize_vision_mxfp8

    n = quantize_vision_mxfp8(v)
    assert isinstance(v.blocks[0].qkv_w, L.MXFP8Weight) and isinstance(v.patch_w, L.MXFP8Weight)
    assert n == 1 + 2 * 4 + 2 * 2
    got, got_d = v(pix, grids)
    assert float((got - ref).norm() / ref.norm()) < 0.1
    assert float((got_d - ref_d).norm() / ref_d.norm()) < 0.1
