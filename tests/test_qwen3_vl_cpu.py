"""Qwen3-VL on CPU (fp32) against HF transformers: image preprocessing, placeholder expansion,
vision encoder with 2-D rotary and DeepStack mergers, interleaved M-RoPE and DeepStack
injection in the text decoder.  Greedy tokens must match HF's full-sequence forward."""
import tempfile

import numpy as np
import pytest
import torch

from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.entrypoints import LLM

IMG, VS, VE = 500, 501, 502  # image pad, vision start, vision end token ids
VID = 503                      # video pad
PROC = {"min_pixels": 16 * 16, "max_pixels": 32 * 32}


def _ckpt():
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration

    torch.manual_seed(0)
    cfg = Qwen3VLConfig(
        text_config=dict(hidden_size=64, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=16, intermediate_size=128, vocab_size=512, max_position_embeddings=512,
                         rope_parameters={"rope_type": "default", "rope_theta": 10000.0,
                                          "mrope_section": [4, 2, 2], "mrope_interleaved": True},
                         initializer_range=0.05, tie_word_embeddings=False),
        vision_config=dict(hidden_size=32, intermediate_size=64, num_heads=2, depth=2, patch_size=4,
                           temporal_patch_size=2, spatial_merge_size=2, out_hidden_size=64,
                           num_position_embeddings=16, deepstack_visual_indexes=[0, 1],
                           initializer_range=0.05),
        image_token_id=IMG, video_token_id=VID, vision_start_token_id=VS, vision_end_token_id=VE,
        tie_word_embeddings=False)
    hf = Qwen3VLForConditionalGeneration(cfg).float().eval()
    with torch.no_grad():
        for n, p in hf.model.visual.named_parameters():
            if "norm" in n and n.endswith("bias"):
                p.normal_(0.0, 0.05)
    d = tempfile.mkdtemp(prefix="tiny_qwen3vl_")
    hf.save_pretrained(d, safe_serialization=True)
    return d, hf


def _hf_greedy(hf, ids, pixels, grid, n):
    ids = list(ids)
    out = []
    with torch.no_grad():
        for _ in range(n):
            t = torch.tensor([ids])
            mm = (t == IMG).int()
            logits = hf(input_ids=t, pixel_values=pixels, image_grid_thw=grid, mm_token_type_ids=mm).logits
            nxt = int(logits[0, -1].argmax())
            out.append(nxt)
            ids.append(nxt)
    return out


def test_qwen3_vl_generate_matches_hf():
    from vllm_neuron_b200.engine.multimodal import _processor

    d, hf = _ckpt()
    rng = np.random.default_rng(0)
    img = (rng.random((24, 16, 3)) * 255).astype(np.uint8)
    prompt = [7, 8, VS, IMG, VE, 9, 10, 11, 12]
    llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=2, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=8, mm_processor_kwargs=PROC, skip_tokenizer_init=True)
    outs = llm.generate([{"prompt_token_ids": prompt, "multi_modal_data": {"image": img}},
                         {"prompt_token_ids": [3, 4, 5, 6]}],
                        SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
    got = outs[0].outputs[0].token_ids
    # HF oracle with the same preprocessing and expansion
    proc = _processor(d, llm.engine.model.cfg.raw["vision_config"], PROC)
    o = proc(images=[img], return_tensors="pt")
    grid = o["image_grid_thw"]
    n_img = int(grid.prod()) // 4
    ids = prompt[:3] + [IMG] * n_img + prompt[4:]
    assert n_img > 1 and len(outs[0].prompt_token_ids) == len(ids)
    ref = _hf_greedy(hf, ids, o["pixel_values"], grid, 6)
    assert got == ref, (got, ref)
    # the text-only request in the same batch is unaffected
    ref_txt = []
    t_ids = [3, 4, 5, 6]
    with torch.no_grad():
        for _ in range(6):
            nxt = int(hf(input_ids=torch.tensor([t_ids])).logits[0, -1].argmax())
            ref_txt.append(nxt)
            t_ids.append(nxt)
    assert outs[1].outputs[0].token_ids == ref_txt


def test_mrope_positions_layout():
    from vllm_neuron_b200.models.qwen3_vl import mrope_positions

    ids = [1, 2, IMG, IMG, IMG, IMG, IMG, IMG, 3]
    pos, delta = mrope_positions(ids, IMG, [(1, 4, 6)], 2)   # 2 x 3 merged grid
    assert pos[:, :2].tolist() == [[0, 1], [0, 1], [0, 1]]
    assert pos[0, 2:8].tolist() == [2] * 6
    assert pos[1, 2:8].tolist() == [2, 2, 2, 3, 3, 3]
    assert pos[2, 2:8].tolist() == [2, 3, 4, 2, 3, 4]
    assert pos[:, 8].tolist() == [5, 5, 5]  # after the image: start + max(h, w) / merge
    assert delta == 6 - 9


@pytest.mark.parametrize("packed", [False, True])
def test_qwen3_vl_video_matches_hf(packed):
    """A 4-frame video (two temporal patch groups, each a timestamp + vision span) next to an
    image: greedy tokens match HF's forward with pixel_values_videos / video_grid_thw.  With
    ``packed`` the encoder runs the image and the video's frame groups packed into 64-row
    blocks (block-local attention bounds)."""
    from vllm_neuron_b200.engine.multimodal import _processor, _video_processor

    d, hf = _ckpt()
    rng = np.random.default_rng(3)
    frames = (rng.random((4, 16, 24, 3)) * 255).astype(np.uint8)
    img = (rng.random((16, 16, 3)) * 255).astype(np.uint8)
    ac = {"vision_neuron_config": {"vision_attention_block_size": 64}} if packed else None
    llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=2, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=16, mm_processor_kwargs=PROC, skip_tokenizer_init=True,
              additional_config=ac)
    vc = llm.engine.model.cfg.raw["vision_config"]
    vo = _video_processor(d, vc, PROC)(videos=[frames], return_tensors="pt", do_sample_frames=False,
                                       video_metadata=[{"fps": 2.0, "total_num_frames": 4}])
    t, h, w = vo["video_grid_thw"][0].tolist()
    n = h * w // 4
    io = _processor(d, vc, PROC)(images=[img], return_tensors="pt")
    n_img = int(io["image_grid_thw"].prod()) // 4
    ts = [90, 91]  # stand-ins for the timestamp text tokens of the two groups
    ids = [7, VS] + [IMG] * n_img + [VE, 8]
    for g in range(t):
        ids += [ts[g], VS] + [VID] * n + [VE]
    ids += [9, 10]
    out = llm.generate([{"prompt_token_ids": ids, "multi_modal_data": {"image": img, "video": frames}}],
                       SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
    got = out[0].outputs[0].token_ids
    ref, cur = [], list(ids)
    with torch.no_grad():
        for _ in range(5):
            x = torch.tensor([cur])
            mm = (x == IMG).int() + 2 * (x == VID).int()
            logits = hf(input_ids=x, pixel_values=io["pixel_values"], image_grid_thw=io["image_grid_thw"],
                        pixel_values_videos=vo["pixel_values_videos"], video_grid_thw=vo["video_grid_thw"],
                        mm_token_type_ids=mm).logits
            nxt = int(logits[0, -1].argmax())
            ref.append(nxt)
            cur.append(nxt)
    assert got == ref, (got, ref)
    assert (llm.engine.model.vision_blocks > 0) == packed


def test_encoder_cache_reuses_identical_images():
    """Two requests with the same image run the vision encoder once (content-hash cache)."""
    d, _ = _ckpt()
    rng = np.random.default_rng(4)
    img = (rng.random((24, 16, 3)) * 255).astype(np.uint8)
    llm = LLM(d, device="cpu", dtype="float32", max_num_seqs=2, max_model_len=256, num_gpu_blocks=64,
              max_num_batched_tokens=64, mm_processor_kwargs=PROC, skip_tokenizer_init=True)
    calls = []
    vis = llm.engine.model.visual
    orig = vis.forward
    vis.forward = lambda *a, **k: (calls.append(1), orig(*a, **k))[1]
    reqs = [{"prompt_token_ids": [7, 8, VS, IMG, VE, 9], "multi_modal_data": {"image": img}},
            {"prompt_token_ids": [3, VS, IMG, VE, 4, 5], "multi_modal_data": {"image": img}}]
    a = llm.generate(reqs, SamplingParams(temperature=0, max_tokens=3, ignore_eos=True))
    assert len(calls) == 1 and llm.engine.runner.encoder_cache_hits == 1
    b = LLM(d, device="cpu", dtype="float32", max_num_seqs=2, max_model_len=256, num_gpu_blocks=64,
            max_num_batched_tokens=64, mm_processor_kwargs=PROC,
            skip_tokenizer_init=True).generate(reqs[1:], SamplingParams(temperature=0, max_tokens=3,
                                                                        ignore_eos=True))
    assert a[1].outputs[0].token_ids == b[0].outputs[0].token_ids
