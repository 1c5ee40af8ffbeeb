"""Packed Qwen3-VL vision encoder on the GPU: CUDA-graph replays of the packed encoder (one
graph per block count) against the per-image encoder, for two different image mixes that share a
bucket (the second one replays the graph captured for the first)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(dev):
    from transformers import Qwen3VLConfig

    from vllm_neuron_b200.config import ModelArchConfig, VisionConfig
    from vllm_neuron_b200.models.qwen3_vl import Qwen3VLForConditionalGeneration

    cfg = Qwen3VLConfig(
        text_config=dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1,
                         head_dim=128, intermediate_size=512, vocab_size=1024, max_position_embeddings=512,
                         rope_parameters={"rope_type": "default", "rope_theta": 10000.0,
                                          "mrope_section": [24, 20, 20], "mrope_interleaved": True}),
        vision_config=dict(hidden_size=256, intermediate_size=512, num_heads=4, depth=3, patch_size=16,
                           temporal_patch_size=2, spatial_merge_size=2, out_hidden_size=256,
                           num_position_embeddings=2304, deepstack_visual_indexes=[0, 2]),
        image_token_id=1000, video_token_id=1001, vision_start_token_id=1002, vision_end_token_id=1003)
    d = cfg.to_dict()
    d["architectures"] = ["Qwen3VLForConditionalGeneration"]
    m = Qwen3VLForConditionalGeneration(ModelArchConfig.from_hf(d), device=dev, dtype=torch.bfloat16,
                                        max_tokens=512)
    m.init_random(0, std=0.05)
    m.configure_vision(VisionConfig.from_dict({"vision_attention_block_size": 512,
                                               "num_vision_tokens_buckets": [1024, 2048]}))
    return m


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def test_packed_encoder_graphs_match_per_image(cuda_device):
    m = _model(cuda_device)
    assert m.vision_graphs
    g = torch.Generator(device="cpu").manual_seed(0)
    for grids in ([(1, 16, 16), (1, 8, 24), (2, 8, 8), (1, 12, 12)],
                  [(1, 20, 20), (1, 4, 8), (1, 8, 8)]):
        n = sum(t * h * w for t, h, w in grids)
        pix = (torch.randn(n, 3 * 2 * 16 * 16, generator=g) * 0.5).to(cuda_device, torch.bfloat16)
        emb, deep = m.encode_images(pix, grids)
        torch.cuda.synchronize()
        ref_e, ref_d = m.visual(pix, grids)
        assert emb.shape == ref_e.shape and deep.shape == ref_d.shape
        assert _rel(emb, ref_e) < 2e-2
        assert _rel(deep, ref_d) < 2e-2
    # both mixes fit two 512-row blocks of the 1024 bucket: one captured graph
    assert list(m._vgraphs) == [(2, 512)]
    assert m.vision_blocks == 4
