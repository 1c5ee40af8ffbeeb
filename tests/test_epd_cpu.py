"""Encoder disaggregation on CPU: rank 0 is an encoder instance running Qwen3-VL's vision
encoder for the image requests and sending the embeddings; rank 1 serves the requests with
those embeddings instead of running its own encoder.  Greedy outputs equal a single engine's."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from tests.test_qwen3_vl_cpu import IMG, PROC, VE, VS, _ckpt

KW = dict(device="cpu", dtype="float32", max_num_seqs=2, max_model_len=256, num_gpu_blocks=64,
          max_num_batched_tokens=8, mm_processor_kwargs=PROC, skip_tokenizer_init=True)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts():
    rng = np.random.default_rng(1)
    imgs = [(rng.random((24, 16, 3)) * 255).astype(np.uint8), (rng.random((16, 32, 3)) * 255).astype(np.uint8)]
    return [{"prompt_token_ids": [7, 8, VS, IMG, VE, 9, 10], "multi_modal_data": {"image": imgs[0]}},
            {"prompt_token_ids": [3, 4, 5, 6]},
            {"prompt_token_ids": [11, VS, IMG, VE, 12], "multi_modal_data": {"image": imgs[1]}}]


def _worker(rank, port, ckpt, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch

    torch.set_num_threads(1)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    try:
        role = "ec_producer" if rank == 0 else "ec_consumer"
        llm = LLM(ckpt, ec_transfer_config={"ec_role": role}, **KW)
        if rank == 0:
            q.put((rank, llm.encode_remote(_prompts())))
        else:
            calls = []
            vis = llm.engine.model.visual
            orig = vis.forward
            vis.forward = lambda *a, **k: (calls.append(1), orig(*a, **k))[1]
            outs = llm.generate(_prompts(), SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
            q.put((rank, ([o.outputs[0].token_ids for o in outs], len(calls))))
    except Exception:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        ps.destroy_parallel_state()


def test_encoder_disaggregation_matches_single_engine():
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    d, _ = _ckpt()
    ref = LLM(d, **KW).generate(_prompts(), SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, d, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in (1, 0):
        assert not isinstance(res[r], str), res[r]
    assert res[0] == 2
    toks, encoder_calls = res[1]
    assert toks == ref, (toks, ref)
    assert encoder_calls == 0  # the serving instance never ran its vision encoder


def _vision_dp_worker(rank, port, ckpt, q, extra=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch

    torch.set_num_threads(1)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    try:
        llm = LLM(ckpt, tensor_parallel_size=2, **dict(KW, **(extra or {})))
        outs = llm.generate(_three_image_prompts(), SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
        q.put((rank, ([o.outputs[0].token_ids for o in outs], llm.engine.model.vision_calls,
                     llm.engine.model.vision_blocks)))
    except Exception:  # pragma: no cover
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        ps.destroy_parallel_state()


def _three_image_prompts():
    rng = np.random.default_rng(2)
    imgs = [(rng.random(s) * 255).astype(np.uint8) for s in ((24, 16, 3), (16, 32, 3), (16, 16, 3))]
    return [{"prompt_token_ids": [7, VS, IMG, VE, 8, VS, IMG, VE, 9, VS, IMG, VE, 10],
             "multi_modal_data": {"image": imgs}}]


def test_vision_data_parallel_over_tp_ranks():
    """TP=2: the request's three images are encoded 2 + 1 by the two ranks and gathered; the
    tokens equal a TP=1 run (which encodes all three itself)."""
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    d, _ = _ckpt()
    ref_llm = LLM(d, **KW)
    ref = ref_llm.generate(_three_image_prompts(), SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    assert ref_llm.engine.model.vision_calls == 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_vision_dp_worker, args=(r, port, d, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    assert res[0][0] == ref and res[1][0] == ref, (res, ref)
    assert res[0][1] == 2 and res[1][1] == 1


def test_vision_tensor_parallel_over_tp_ranks():
    """Vision TP=2 on TP=2: each rank holds half of every encoder block's heads and MLP
    (all-reduced row-parallel projections); both ranks encode all three images together and
    the tokens equal the TP=1 run."""
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    d, _ = _ckpt()
    ref = LLM(d, **KW).generate(_three_image_prompts(),
                                SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    extra = {"additional_config": {"neuron_config": {"vision_tp_size": 2}}}
    procs = [ctx.Process(target=_vision_dp_worker, args=(r, port, d, q, extra)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    assert res[0][0] == ref and res[1][0] == ref, (res, ref)
    assert res[0][1] == 3 and res[1][1] == 3


@pytest.mark.parametrize("vision", [{"vision_attention_block_size": 32},
                                    {"vision_attention_block_size": 32, "tp_size": 2}])
def test_packed_vision_over_tp_ranks(vision):
    """Packed encoder on TP=2: the three images (32, 24 and 16 patches) take three 32-row
    blocks, padded to four for two replicas; with vision DP (default) each rank encodes two blocks and the merged
    rows are all-gathered; with vision TP 2 both ranks encode the three blocks on half the heads.
    Tokens equal the unpacked TP=1 run."""
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    d, _ = _ckpt()
    ref = LLM(d, **KW).generate(_three_image_prompts(),
                                SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    extra = {"additional_config": {"vision_neuron_config": vision}}
    procs = [ctx.Process(target=_vision_dp_worker, args=(r, port, d, q, extra)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    assert res[0][0] == ref and res[1][0] == ref, (res, ref)
    blocks = 3 if vision.get("tp_size", 1) == 2 else 2  # no DP replicas: no padding
    assert res[0][2] == blocks and res[1][2] == blocks


def _cdp_vl_worker(rank, port, ckpt, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch

    torch.set_num_threads(1)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    try:
        llm = LLM(ckpt, tensor_parallel_size=1, **dict(KW, additional_config={"neuron_config": {
            "attention_dp_size": 2, "embedding_dp_size": 2, "lm_head_dp_size": 2}}))
        prompts = _three_image_prompts() * 2  # two image requests: one per replica
        outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
        q.put((rank, [o.outputs[0].token_ids for o in outs]))
    except Exception:  # pragma: no cover
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        ps.destroy_parallel_state()


def test_component_dp_vision_language():
    """Qwen3-VL with attention / embedding / LM-head DP over two replicas (each encodes its own
    requests' images; image rows replace the gathered embedding on the replica): tokens equal
    the single-process run."""
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    d, _ = _ckpt()
    prompts = _three_image_prompts() * 2
    ref = LLM(d, **KW).generate(prompts, SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_cdp_vl_worker, args=(r, port, d, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
        assert res[r] == ref, (res, ref)
