"""Bucket utilities (power-of-two generation, validation, bucket lookup, decode-graph buckets)
and their wiring: ``num_seqs_buckets`` selects the decode CUDA graphs the runner captures."""
import pytest

from vllm_neuron_b200.utils import buckets as B


def test_pow2_and_lookup():
    assert B.pow2_buckets(1, 100) == [1, 2, 4, 8, 16, 32, 64, 100]
    assert B.pow2_buckets(3, 16) == [4, 8, 16]
    assert B.pow2_buckets(8, 8) == [8]
    with pytest.raises(ValueError):
        B.pow2_buckets(0, 4)
    bk = [4, 8, 16]
    assert [B.bucket_for(bk, n) for n in (1, 4, 5, 16, 17)] == [4, 4, 8, 16, 17]
    assert B.bucket_for(None, 9) == 9


def test_validate_and_decode_graph_buckets():
    assert B.validate_buckets([8, 2, 8, 4], "x") == [2, 4, 8]
    for bad in ([0, 2], [2, -1], [1.5], [True]):
        with pytest.raises(ValueError):
            B.validate_buckets(bad, "x")
    with pytest.raises(ValueError):
        B.validate_buckets([2, 64], "x", max_value=32)
    assert B.decode_graph_buckets(40) == [1, 2, 4, 8, 16, 24, 32, 40]
    assert B.decode_graph_buckets(64, [3, 17, 200]) == [3, 17, 64]
    assert B.decode_graph_buckets(0) == []


def test_runner_uses_num_seqs_buckets():
    from tests._tiny import tiny_llama_checkpoint
    from vllm_neuron_b200.entrypoints import LLM

    ckpt, _ = tiny_llama_checkpoint()
    llm = LLM(ckpt, device="cpu", dtype="float32", max_num_seqs=16, max_model_len=64, num_gpu_blocks=32,
              max_num_batched_tokens=32, additional_config={"neuron_config": {"num_seqs_buckets": [2, 6, 12]}})
    assert llm.engine.runner.graph_buckets == [2, 6, 12, 16]
