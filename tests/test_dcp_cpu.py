"""Decode context parallelism: token-sharded KV with LSE-merged partials (CPU oracle paths).

Every DCP rank holds one block_size slice of each (dcp * block_size) token window; the
partials of all ranks, merged by log-sum-exp, must equal attention over the whole sequence
(reference: docs/design/parallelism/dcp.md; functional/attention/attention_decode.py:902-1062).
"""
import numpy as np
import pytest
import torch

from vllm_neuron_b200 import ops
from vllm_neuron_b200.ops.attention import dcp_local_count


@pytest.mark.parametrize("bs,dcp", [(16, 2), (16, 4), (8, 3)])
def test_local_count_partitions_positions(bs, dcp):
    for n in [0, 1, 5, bs, bs + 1, 2 * bs * dcp + 3, 1000]:
        counts = [dcp_local_count(n, bs, dcp, r) for r in range(dcp)]
        assert sum(counts) == n
        # brute force: owner of position p is (p // bs) % dcp
        for r in range(dcp):
            assert counts[r] == sum(1 for p in range(n) if (p // bs) % dcp == r)


def shard_cache(k_full, v_full, seq_lens, bs, dcp, blocks_per_seq):
    """Split whole-sequence K/V [B, Hkv, L, D] into per-rank paged caches (virtual block v of a
    sequence -> local block id 1 + b * blocks_per_seq + v on every rank)."""
    B, Hkv, Lmax, D = k_full.shape
    nblk = 1 + B * blocks_per_seq
    caches = []
    for r in range(dcp):
        kc = torch.zeros(nblk, Hkv, bs, D)
        vc = torch.zeros(nblk, Hkv, bs, D)
        local = []
        for b in range(B):
            L = seq_lens[b]
            pos = [p for p in range(L) if (p // bs) % dcp == r]
            local.append(len(pos))
            for j, p in enumerate(pos):
                blk = 1 + b * blocks_per_seq + j // bs
                kc[blk, :, j % bs] = k_full[b, :, p]
                vc[blk, :, j % bs] = v_full[b, :, p]
        caches.append((kc, vc, local))
    bt = torch.tensor([[1 + b * blocks_per_seq + v for v in range(blocks_per_seq)]
                       for b in range(B)], dtype=torch.int32)
    return caches, bt


def full_cache(k_full, v_full, bs, blocks_per_seq):
    B, Hkv, Lmax, D = k_full.shape
    kc = torch.zeros(1 + B * blocks_per_seq, Hkv, bs, D)
    vc = torch.zeros_like(kc)
    for b in range(B):
        for p in range(Lmax):
            blk = 1 + b * blocks_per_seq + p // bs
            kc[blk, :, p % bs] = k_full[b, :, p]
            vc[blk, :, p % bs] = v_full[b, :, p]
    bt = torch.tensor([[1 + b * blocks_per_seq + v for v in range(blocks_per_seq)]
                       for b in range(B)], dtype=torch.int32)
    return kc, vc, bt


@pytest.mark.parametrize("q_lens,seq_lens,dcp", [
    ([1, 1, 1], [37, 64, 5], 2),        # decode
    ([1, 1], [100, 17], 4),
    ([20, 1, 7], [20, 90, 40], 2),      # prefill chunks (first and continued) + decode
])
def test_dcp_partials_merge_to_full_attention(q_lens, seq_lens, dcp):
    torch.manual_seed(0)
    bs, Hkv, G, D = 16, 1, 4, 32
    Hq = Hkv * G
    B = len(seq_lens)
    Lmax = max(seq_lens)
    bps = (Lmax + bs - 1) // bs
    k_full = torch.randn(B, Hkv, Lmax, D)
    v_full = torch.randn(B, Hkv, Lmax, D)
    T = sum(q_lens)
    q = torch.randn(T, Hq, D)
    q_start = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    scale = D ** -0.5

    kc, vc, bt_full = full_cache(k_full, v_full, bs, bps)
    want = ops.paged_attention_ref(q, kc, vc, bt_full, sl, q_start, scale)

    caches, bt = shard_cache(k_full, v_full, seq_lens, bs, dcp, bps)
    po = torch.empty(dcp, T, Hq, D)
    pl = torch.empty(dcp, T, Hq)
    for r, (kcr, vcr, local) in enumerate(caches):
        ops.paged_attention_partial(q, kcr, vcr, bt, torch.tensor(local, dtype=torch.int32),
                                    q_start, torch.zeros(0, 2, dtype=torch.int32), False, 1,
                                    scale, po[r:r + 1], pl[r:r + 1], dcp_seq_lens=sl,
                                    dcp_size=dcp, dcp_rank=r)
    got = ops.attn_combine(po, pl, torch.empty(T, Hq, D))
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)


def test_dcp_slot_mapping_and_block_tables():
    """The model runner writes a token only on its owning rank, at the local slot of its
    virtual block (scheduler blocks hold dcp * block_size tokens)."""
    from vllm_neuron_b200.worker.model_runner import dcp_slots
    bs, dcp = 4, 2
    positions = np.arange(0, 19)
    vblocks = np.array([7, 3, 9])  # scheduler block ids of one sequence (8 tokens each)
    for r in range(dcp):
        slots = dcp_slots(positions, vblocks[positions // (bs * dcp)], bs, dcp, r)
        for p, s in zip(positions, slots):
            owner = (p // bs) % dcp
            if owner != r:
                assert s == -1
            else:
                assert s == vblocks[p // (bs * dcp)] * bs + p % bs


def _dcp_worker(rank, world, port, ckpt, prompts, q, dcp):
    import os

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel import state as ps

    try:
        llm = LLM(ckpt, tensor_parallel_size=world, device="cpu", max_num_seqs=8,
                  max_model_len=128, num_gpu_blocks=24, max_num_batched_tokens=40, block_size=4,
                  decode_context_parallel_size=dcp)
        outs = llm.generate(prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
        q.put((rank, ([o.outputs[0].token_ids for o in outs], llm.engine.runner.block_size,
                      llm.engine.runner.cache_block_size)))
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, repr(e) + traceback.format_exc()))
    finally:
        ps.destroy_parallel_state()


def test_dcp2_engine_matches_tp1():
    """Two gloo ranks (TP=2 over one replicated KV head, DCP=2): each rank keeps half of every
    sequence's KV (chunked prefill over 4-token cache blocks, then decode); greedy tokens equal
    the single-rank engine's."""
    import multiprocessing as mp
    import socket

    from tests._tiny import random_prompts, tiny_llama_checkpoint
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM

    ckpt, _ = tiny_llama_checkpoint(num_key_value_heads=1)
    prompts = random_prompts(n=3, length=23, seed=3)
    ref = LLM(ckpt, device="cpu", max_num_seqs=8, max_model_len=128, num_gpu_blocks=64,
              max_num_batched_tokens=40, block_size=4).generate(
        prompts, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    ref = [o.outputs[0].token_ids for o in ref]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dcp_worker, args=(r, 2, port, ckpt, prompts, q, 2)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        toks, sched_bs, cache_bs = res[r]
        assert (sched_bs, cache_bs) == (8, 4)
        assert toks == ref, (r, toks, ref)


def test_dcp_validation():
    from vllm_neuron_b200.config import ModelArchConfig
    from vllm_neuron_b200.engine.llm_engine import validate_dcp
    from vllm_neuron_b200.parallel.comm import EmulatedRankComm

    class M:
        supports_dcp = True

    arch = ModelArchConfig.from_hf(dict(architectures=["LlamaForCausalLM"], hidden_size=256,
                                        num_hidden_layers=1, num_attention_heads=8,
                                        num_key_value_heads=2, intermediate_size=512,
                                        vocab_size=128, max_position_embeddings=256))
    validate_dcp(arch, M(), EmulatedRankComm(8), 4)   # TP 8 over 2 KV heads: sets of 4 share one
    with pytest.raises(ValueError):
        validate_dcp(arch, M(), EmulatedRankComm(2), 2)   # TP 2 = KV heads: nothing replicated
    with pytest.raises(ValueError):
        validate_dcp(arch, M(), EmulatedRankComm(8), 8)   # a set would span two KV heads
    M.supports_dcp = False
    with pytest.raises(NotImplementedError):
        validate_dcp(arch, M(), EmulatedRankComm(8), 2)
