"""Model runner: batch preparation, KV-cache ownership, CUDA graphs and on-device sampling.

Per step the host builds every int/float input of the forward pass and of the sampler in
ONE pinned int32 buffer (floats are stored as their bit patterns), copies it to the device
with one ``cudaMemcpyAsync``, and views the sections on the device.  Pure-decode batches
replay a CUDA graph captured per batch-size bucket (padded rows write nothing to the cache:
slot -1, null block 0); prefill and mixed batches run eagerly.  The sampled token ids come
back with one device->host copy into pinned memory.

Reference: NeuronModelRunner (vllm_neuron/vllm/worker/neuron_model_runner.py): input prep
:2605-3057, attention metadata :4084-4258, KV cache allocation :8456-8619, per-bucket graph
compile + warm-up :4437-5094 (CUDA graphs per bucket here), on-device sampling :5717-6054.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass

import numpy as np
import torch

from .. import envs, ops
from ..exceptions import KVCacheBudgetError
from ..engine.scheduler import SchedulerOutput
from ..models.llama import ForwardBatch

_ALIGN = 4  # int32 elements (16 bytes) between sections


def _round(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def dcp_slots(positions: np.ndarray, vblocks: np.ndarray, block_size: int, dcp_size: int,
              dcp_rank: int) -> np.ndarray:
    """KV-write slots of one DCP rank: scheduler blocks hold ``dcp_size * block_size`` tokens
    and every rank keeps its ``block_size`` slice of each in its own cache block of the same id;
    positions owned by another rank get -1 (no write).  ``vblocks``: the scheduler block of each
    position (reference: CP-aware slot mapping, docs/design/parallelism/dcp.md)."""
    off = positions % (block_size * dcp_size)
    own = (off // block_size) == dcp_rank
    return np.where(own, vblocks * block_size + off % block_size, -1).astype(np.int32)


@dataclass
class Layout:
    """Section offsets (int32 elements) inside the packed input buffer."""

    T: int
    B: int
    S: int
    W: int
    nblk: int

    def __post_init__(self):
        o = 0
        self.off = {}
        for name, n in (("ids", self.T), ("pos", self.T), ("slot", self.T), ("qstart", self.B + 1),
                        ("seqlen", self.B), ("lseqlen", self.B), ("lidx", self.S), ("work", 2 * self.W),
                        ("bt", self.B * self.nblk), ("temp", self.S), ("topk", self.S),
                        ("topp", self.S), ("minp", self.S), ("seed", 2 * self.S), ("offs", self.S),
                        ("rslot", self.S), ("sslot", self.B), ("nsplit", 1)):
            self.off[name] = (o, n)
            o += _round(n)
        self.total = o


class ModelRunner:
    def __init__(self, model, *, max_num_seqs: int, max_num_batched_tokens: int, max_model_len: int,
                 block_size: int = 16, cuda_graphs: bool = True, graph_buckets: list[int] | None = None,
                 device="cuda", seed: int = 0):
        self.model = model
        self.sampling_dp = False   # sampling data parallelism over the TP group (see _sample_dp)
        self.encoder_cache_size = 32  # vision encodings kept for reuse (see _encode_cached)
        self.sampling_dp_steps = 0
        self.device = torch.device(device)
        self.is_cuda = self.device.type == "cuda"
        self.max_num_seqs = max_num_seqs
        self.max_tokens = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.block_size = block_size
        self.max_blocks = (max_model_len + block_size - 1) // block_size
        # Decode context parallelism: scheduler blocks of block_size tokens, of which this rank
        # keeps the dcp_rank-th slice of cache_block_size tokens (see set_dcp)
        self.dcp_size, self.dcp_rank, self.cache_block_size = 1, 0, block_size
        self.use_graphs = cuda_graphs and self.is_cuda and not envs.VLLM_B200_DISABLE_CUDA_GRAPHS
        self._last_prefill_rows = ops.attention.PREFILL_ROWS  # rows per prefill work item
        from ..utils.buckets import decode_graph_buckets

        cap = min(max_num_seqs, model.max_decode_tokens)
        self.graph_buckets = decode_graph_buckets(cap, graph_buckets)
        self.graphs: dict[int, tuple] = {}
        self.seed = seed
        self.num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count if self.is_cuda else 148
        # logits rows: one per sampling request, or 1 + drafts for verified requests (<= tokens)
        max_layout = Layout(self.max_tokens, max_num_seqs, max(max_num_seqs, self.max_tokens), self._max_work(),
                            self.max_blocks)
        pin = self.is_cuda
        # Two pinned input buffers and two pinned output buffers: with asynchronous
        # scheduling, step N+1 is packed while step N's copies may still be in flight.
        self.host_bufs = [torch.zeros(max_layout.total, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self.host_buf = self.host_bufs[0]
        self.host_np = self.host_buf.numpy()
        self._buf_idx = 0
        self.dev_buf = torch.zeros(max_layout.total, dtype=torch.int32, device=self.device)
        self.tok_hosts = [torch.zeros(max_num_seqs, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self.lp_hosts = [torch.zeros(max_num_seqs, dtype=torch.float32, pin_memory=pin) for _ in range(2)]
        self.rank_hosts = [torch.zeros(max_num_seqs, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self.tok_host, self.lp_host = self.tok_hosts[0], self.lp_hosts[0]
        # Device-resident last sampled token of every request slot (async decode inputs).
        self.max_slots = 2 * max_num_seqs + 8
        self.pad_slot = self.max_slots - 1
        self.last_tok = torch.zeros(self.max_slots, dtype=torch.int32, device=self.device)
        self.tok_dev = torch.zeros(max_num_seqs, dtype=torch.int32, device=self.device)
        self.lp_dev = torch.zeros(max_num_seqs, dtype=torch.float32, device=self.device)
        self.rank_dev = torch.zeros(max_num_seqs, dtype=torch.int32, device=self.device)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.num_graph_replays = 0
        self.num_eager_steps = 0
        self.graph_kernels: dict[int, int] = {}  # kernels recorded per captured bucket
        self.replayed_kernels = 0
        self.kv_cache = None
        # Snapshot capture of selected steps' packed inputs (snapshot/: VLLM_B200_SNAPSHOT_*;
        # reference: vllm_neuron/snapshot/*, runtime input capture).
        from ..snapshot import SnapshotCapturer, SnapshotConfig

        tp = getattr(model, "tp", None)
        self.snapshot = SnapshotCapturer(SnapshotConfig.from_env(), rank=getattr(tp, "rank", 0),
                                         world=getattr(tp, "world", 1))
        self.snapshot_dir = self.snapshot.cfg.directory if self.snapshot.enabled else None

    def set_dcp(self, size: int, rank: int):
        """Shard every sequence's KV over a DCP replica set of ``size`` ranks: the scheduler's
        blocks (``self.block_size`` tokens) are split into ``size`` slices of the model's cache
        block, and this rank writes and attends over slice ``rank`` only."""
        if self.block_size % size:
            raise ValueError("the scheduler block size must be a multiple of the DCP size")
        self.dcp_size, self.dcp_rank = int(size), int(rank)
        self.cache_block_size = self.block_size // size
        self.use_graphs = False  # DCP steps run eagerly (their collectives are not captured)

    def _group(self) -> int:
        """Packed query rows per KV head: the local heads, times the DCP set (Q is gathered)."""
        return max(1, self.model.Hq // self.model.Hkv) * self.dcp_size

    def _max_work(self) -> int:
        # prefill work items: ceil(q_len * G / 64) per sequence, bounded by tokens*G/64 + seqs
        G = self._group()
        return self.max_tokens * G // ops.attention.PREFILL_ROWS + self.max_num_seqs + 1

    # ------------------------------------------------------------------ KV cache
    def kv_bytes_per_block(self) -> int:
        return self.model.kv_bytes_per_block()

    def allocate_kv_cache(self, num_blocks: int):
        m = self.model
        n_kv = getattr(m, "num_kv_layers", m.cfg.num_layers)
        shape = (n_kv, 2) + m.kv_cache_shape(num_blocks)
        self.kv_cache = torch.zeros(shape, dtype=getattr(m, "kv_dtype", m.dtype), device=self.device)
        m.bind_kv_cache([(self.kv_cache[i, 0], self.kv_cache[i, 1]) for i in range(n_kv)])
        self.num_blocks = num_blocks

    def profile_num_blocks(self, gpu_memory_utilization: float, reserve_bytes: int = 2 << 30) -> int:
        """Blocks that fit in ``utilization * total`` after weights and workspaces."""
        if not self.is_cuda:
            return 4096
        torch.cuda.synchronize(self.device)
        free, total = torch.cuda.mem_get_info(self.device)
        used = total - free
        budget = total * gpu_memory_utilization - used - reserve_bytes
        cap = envs.VLLM_B200_KV_CACHE_MAX_GIB
        if cap is not None:
            budget = min(budget, cap * 2**30)
        if budget < (envs.VLLM_B200_MIN_KV_BUDGET_GIB or 0.0) * 2**30:
            raise KVCacheBudgetError(f"KV-cache budget {budget / 2**30:.2f} GiB is below "
                                     f"VLLM_B200_MIN_KV_BUDGET_GIB={envs.VLLM_B200_MIN_KV_BUDGET_GIB}")
        n = int(budget // self.kv_bytes_per_block())
        if n < 2:
            raise KVCacheBudgetError(f"not enough memory for the KV cache (budget {budget / 2**30:.2f} GiB)")
        return n

    # ------------------------------------------------------------------ input packing
    def _pack(self, out: SchedulerOutput, lay: Layout, pad_B: int | None = None) -> tuple[int, bool, int]:
        """Fill the pinned buffer for ``out``.  Returns (#sampling rows, decode?, num_splits)."""
        h = self.host_np
        o = lay.off
        sch = out.scheduled
        B = len(sch)
        Bp = pad_B or B
        m = self.model
        bs = self.block_size
        ids = h[o["ids"][0]:o["ids"][0] + lay.T]
        pos = h[o["pos"][0]:o["pos"][0] + lay.T]
        slot = h[o["slot"][0]:o["slot"][0] + lay.T]
        qst = h[o["qstart"][0]:o["qstart"][0] + Bp + 1]
        sl = h[o["seqlen"][0]:o["seqlen"][0] + Bp]
        lsl = h[o["lseqlen"][0]:o["lseqlen"][0] + Bp]
        dcp = self.dcp_size
        bt = h[o["bt"][0]:o["bt"][0] + Bp * lay.nblk].reshape(Bp, lay.nblk)
        lidx = h[o["lidx"][0]:o["lidx"][0] + lay.S]
        t = 0
        s = 0
        q_lens = np.zeros(Bp, dtype=np.int64)
        temp = h[o["temp"][0]:o["temp"][0] + lay.S].view(np.float32)
        topk = h[o["topk"][0]:o["topk"][0] + lay.S]
        topp = h[o["topp"][0]:o["topp"][0] + lay.S].view(np.float32)
        minp = h[o["minp"][0]:o["minp"][0] + lay.S].view(np.float32)
        seed = h[o["seed"][0]:o["seed"][0] + 2 * lay.S].view(np.int64)
        offs = h[o["offs"][0]:o["offs"][0] + lay.S]
        rslot = h[o["rslot"][0]:o["rslot"][0] + lay.S]
        sslot = h[o["sslot"][0]:o["sslot"][0] + Bp]
        for i, sr in enumerate(sch):
            req = sr.req
            n = sr.num_tokens
            st = sr.start
            P = req.num_prompt_tokens
            known = P + len(req.output_token_ids)
            if sr.spec:
                # the last known token, then the drafts being verified
                ids[t] = req.token_at(st)
                ids[t + 1:t + n] = sr.spec
            elif st + n > known:
                # the last input token was sampled by a step still in flight: it is read on
                # the device from the request's slot (id = -(slot + 1))
                nk = max(0, known - st)
                if nk:
                    ids[t:t + nk] = (req.prompt_token_ids + req.output_token_ids)[st:st + nk]
                ids[t + nk:t + n] = -(req.slot + 1)
            elif st >= P:
                ids[t:t + n] = req.output_token_ids[st - P:st - P + n]
            elif st + n <= P:
                ids[t:t + n] = req.prompt_token_ids[st:st + n]
            else:
                ids[t:t + n] = (req.prompt_token_ids + req.output_token_ids)[st:st + n]
            p = np.arange(st, st + n, dtype=np.int32)
            pos[t:t + n] = p
            mm = req.mm
            if mm is not None:  # M-RoPE: temporal position in the prompt, index + delta after it
                P_mm = mm.positions3.shape[1]
                pos[t:t + n] = np.where(p < P_mm, mm.positions3[0, np.minimum(p, P_mm - 1)], p + mm.delta)
            blocks = np.asarray(req.block_ids, dtype=np.int32)
            if dcp > 1:
                cbs = self.cache_block_size
                slot[t:t + n] = dcp_slots(p, blocks[p // bs], cbs, dcp, self.dcp_rank)
                lsl[i] = ops.dcp_local_count(st + n, cbs, dcp, self.dcp_rank)
            else:
                slot[t:t + n] = blocks[p // bs] * bs + (p % bs)
            qst[i] = t
            sl[i] = st + n
            q_lens[i] = n
            sslot[i] = req.slot
            nb = len(req.block_ids)
            bt[i, :nb] = blocks
            bt[i, nb:] = 0
            t += n
            nl = sr.num_logits
            for j in range(nl):
                lidx[s] = t - nl + j
                sp = req.sampling_params
                temp[s] = 0.0 if sp.greedy else sp.temperature
                topk[s] = sp.top_k or 0
                topp[s] = sp.top_p if sp.top_p is not None else 1.0
                minp[s] = sp.min_p or 0.0
                seed[s] = sp.seed if sp.seed is not None else (hash(req.request_id) ^ self.seed) & 0x7FFFFFFFFFFF
                offs[s] = len(req.output_token_ids) + req.num_pending
                rslot[s] = req.slot
                s += 1
        # padding rows (graph buckets): one token each, no cache write, null block
        for i in range(B, Bp):
            ids[t] = 0
            pos[t] = 0
            slot[t] = -1
            qst[i] = t
            sl[i] = 1
            lsl[i] = 1 if self.dcp_rank == 0 else 0
            q_lens[i] = 1
            bt[i, :] = 0
            sslot[i] = self.pad_slot
            lidx[s] = t
            temp[s] = 0.0
            topk[s] = 0
            topp[s] = 1.0
            minp[s] = 0.0
            seed[s] = 0
            offs[s] = 0
            rslot[s] = self.pad_slot
            t += 1
            s += 1
        qst[Bp] = t
        G = self._group()
        if pad_B is not None:
            w = ops.build_work(np.ones(Bp, dtype=np.int64), np.full(Bp, self.max_model_len), G, m.Hkv, self.num_sms,
                               max_splits=m.attn_splits_max, head_dim=m.D)
            # the graph was captured for max_model_len: split this step by its real contexts
            real = ops.build_work(np.ones(Bp, dtype=np.int64), np.maximum(sl[:Bp], 1).astype(np.int64), G, m.Hkv,
                                  self.num_sms, max_splits=m.attn_splits_max, head_dim=m.D)
            h[o["nsplit"][0]] = min(real.num_splits, w.num_splits)
        else:
            kv_lens = (lsl if dcp > 1 else sl)[:Bp].astype(np.int64)
            rows = ops.attention.prefill_rows(m.D, getattr(m, "kv_dtype", None), getattr(m, "block_size", 0),
                                              G, dcp)
            w = ops.build_work(q_lens[:Bp], kv_lens, G, m.Hkv, self.num_sms,
                               max_splits=m.attn_splits_max, head_dim=m.D, prefill_rows=rows)
            self._last_prefill_rows = rows
            h[o["nsplit"][0]] = w.num_splits
        work = h[o["work"][0]:o["work"][0] + 2 * len(w.work)]
        work[:] = w.work.reshape(-1)
        self._last_work_len = len(w.work)
        self._last_max_q = int(q_lens[:Bp].max()) if Bp and pad_B is None else 1
        return s, w.decode, w.num_splits

    def _attach_prompt_embeds(self, out: SchedulerOutput, fb: ForwardBatch):
        """Rows of this step that are prompt positions of requests with ``prompt_embeds``, and
        the image-token rows of vision-language requests (vision embeddings, DeepStack
        features and 3-D M-RoPE positions; the vision encoder runs on a request's first
        chunk and its output is kept until the prompt is prefilled)."""
        rows, parts = [], []
        drows, dparts = [], []
        need3 = False
        t = 0
        for sr in out.scheduled:
            req = sr.req
            emb = req.prompt_embeds
            if emb is not None and sr.start < req.num_prompt_tokens:
                end = min(sr.start + sr.num_tokens, req.num_prompt_tokens)
                rows.extend(range(t, t + end - sr.start))
                parts.append(emb[sr.start:end])
            mm = req.mm
            if mm is not None and sr.start < req.num_prompt_tokens:
                end = min(sr.start + sr.num_tokens, req.num_prompt_tokens)
                sel = mm.image_rows[(mm.image_rows >= sr.start) & (mm.image_rows < end)]
                if len(sel):
                    need3 = True
                    if mm.emb is None:
                        mm.emb, mm.deep = self._encode_cached(mm)
                    idx = torch.as_tensor([mm.row_of[int(r)] for r in sel], device=mm.emb.device)
                    brows = [t + int(r) - sr.start for r in sel]
                    rows.extend(brows)
                    parts.append(mm.emb.index_select(0, idx))
                    if mm.deep is not None and mm.deep.shape[0]:
                        drows.extend(brows)
                        dparts.append(mm.deep.index_select(1, idx))
                if end >= req.num_prompt_tokens:  # prompt done: release the encoder cache
                    mm.emb = mm.deep = None
            t += sr.num_tokens
        pos3 = None
        if need3:  # 3-D positions of every row of the step
            pos3 = np.zeros((t, 3), dtype=np.int32)
            t = 0
            for sr in out.scheduled:
                p = np.arange(sr.start, sr.start + sr.num_tokens)
                mm = sr.req.mm
                if mm is None:
                    pos3[t:t + sr.num_tokens] = p[:, None]
                else:
                    P_mm = mm.positions3.shape[1]
                    inside = p < P_mm
                    pos3[t:t + sr.num_tokens] = np.where(inside[:, None], mm.positions3[:, np.minimum(p, P_mm - 1)].T,
                                                         (p + mm.delta)[:, None])
                t += sr.num_tokens
        if rows:
            order = np.argsort(rows, kind="stable")
            fb.embed_rows = torch.tensor(np.asarray(rows)[order], dtype=torch.long).to(self.device, non_blocking=True)
            cat = torch.cat([x.to(self.device) for x in parts], 0)
            fb.embeds = cat.index_select(0, torch.as_tensor(order, device=cat.device))
        if drows:
            fb.deep_rows = torch.tensor(drows, dtype=torch.long).to(self.device, non_blocking=True)
            fb.deep_feats = torch.cat(dparts, 1)
        if pos3 is not None:
            fb.positions3 = torch.from_numpy(np.ascontiguousarray(pos3)).to(self.device, non_blocking=True)

    def _snapshot(self, out: SchedulerOutput, lay: Layout, decode: bool, splits: int):
        """Save one step's device inputs (the packed int32 buffer and its layout) when the
        snapshot configuration selects it (snapshot/capture.py)."""
        self.snapshot.pre_execute(out, lay, self.host_buf, decode, splits, getattr(self, "_last_work_len", 0),
                                  self.model, self._last_prefill_rows)

    def _views(self, buf: torch.Tensor, lay: Layout, B: int, S: int, W: int, decode: bool, splits: int) -> tuple:
        o = lay.off

        def sec(name, n, dtype=None):
            a = buf[o[name][0]:o[name][0] + n]
            return a.view(dtype) if dtype is not None else a

        nb = lay.nblk
        fb = ForwardBatch(
            input_ids=sec("ids", lay.T), positions=sec("pos", lay.T), slot_mapping=sec("slot", lay.T),
            block_tables=sec("bt", B * nb).view(B, nb), seq_lens=sec("seqlen", B),
            q_start=sec("qstart", B + 1), work=sec("work", 2 * W).view(W, 2),
            logits_indices=sec("lidx", S),
            decode=decode, num_splits=splits, num_tokens=lay.T)
        fb.max_q_len = 1 if decode else getattr(self, "_last_max_q", 0)
        fb.splits_dev = sec("nsplit", 1) if decode and buf.is_cuda else None
        fb.seq_slots = sec("sslot", B)
        if self.dcp_size > 1:
            fb.seq_lens_local = sec("lseqlen", B)
        samp = dict(temperature=sec("temp", S, torch.float32), top_k=sec("topk", S),
                    top_p=sec("topp", S, torch.float32), min_p=sec("minp", S, torch.float32),
                    seeds=sec("seed", 2 * S).view(torch.int64), offsets=sec("offs", S),
                    row_slots=sec("rslot", S))
        fb.last_tok = self.last_tok
        return fb, samp

    def _forward_and_sample(self, fb: ForwardBatch, samp: dict, S: int, tok_out: torch.Tensor,
                            lp_out: torch.Tensor | None, bitmask: torch.Tensor | None = None,
                            rank_out: torch.Tensor | None = None):
        tp = getattr(self.model, "tp", None)
        if (self.sampling_dp and bitmask is None and rank_out is None and tp is not None and tp.world > 1
                and tp.group is not None):
            return self._sample_dp(fb, samp, S, tok_out, lp_out)
        logits = self.model.forward(fb)
        if bitmask is not None:
            ops.sampling.apply_token_bitmask(logits, bitmask)
        ops.sample(logits, samp["temperature"], samp["top_k"], samp["top_p"], samp["seeds"],
                   samp["offsets"], min_p=samp["min_p"], out=tok_out[:S],
                   out_logprob=lp_out[:S] if lp_out is not None else None,
                   row_slots=samp["row_slots"], last_tok=self.last_tok)
        if rank_out is not None:
            # vLLM's logprob semantics: the sampled token's 1-based rank and its log-probability
            # under the raw model distribution (before temperature / top-k / top-p)
            lg = logits[:S].float()
            sel = lg.gather(1, tok_out[:S].long()[:, None])
            rank_out[:S].copy_((lg > sel).sum(1) + 1)
            if lp_out is not None:
                lp_out[:S].copy_((sel[:, 0] - torch.logsumexp(lg, dim=1)))

    def _sample_dp(self, fb: ForwardBatch, samp: dict, S: int, tok_out: torch.Tensor,
                   lp_out: torch.Tensor | None):
        """Sampling data parallelism over the TP group: the LM head's vocab-sharded logits
        ``[S, V/W]`` are exchanged by one all-to-all into ``[S/W, V]`` row blocks, each rank
        samples its rows, and the tokens (and logprobs) are all-gathered.  Rows sample with
        their own seeds, so the tokens equal the replicated path's.  Reference: sampling DP,
        the sampling all-to-all / gather groups (vllm_neuron/parallel/neuron_parallel_state.py:
        116-133,546-574; functional/topk.py:222-322)."""
        import torch.distributed as dist

        m = self.model
        tp = m.tp
        W, r = tp.world, tp.rank
        m.skip_logits_gather = True
        try:
            local = m.forward(fb)                                 # [S, V_local]
        finally:
            m.skip_logits_gather = False
        Vl = local.shape[1]
        per = -(-S // W)
        send = torch.zeros(W * per, Vl, dtype=local.dtype, device=local.device)
        send[:S] = local[:S]
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=tp.group)        # block w: rows of rank r, vocab shard w
        mine = recv.view(W, per, Vl).permute(1, 0, 2).reshape(per, W * Vl)[:, :m.V]

        def rows(t):
            p = torch.zeros(W * per, dtype=t.dtype, device=t.device)
            p[:S] = t[:S]
            return p[r * per:(r + 1) * per]

        mp = {k: rows(samp[k]) for k in ("temperature", "top_k", "top_p", "min_p", "offsets")}
        seeds = torch.zeros(W * per, dtype=samp["seeds"].dtype, device=samp["seeds"].device)
        seeds[:S] = samp["seeds"][:S]
        tok = torch.empty(per, dtype=torch.int32, device=local.device)
        lp = torch.empty(per, dtype=torch.float32, device=local.device) if lp_out is not None else None
        ops.sample(mine, mp["temperature"], mp["top_k"], mp["top_p"], seeds[r * per:(r + 1) * per],
                   mp["offsets"], min_p=mp["min_p"], out=tok, out_logprob=lp)
        tok_out[:S].copy_(tp.all_gather(tok, dim=0)[:S])
        if lp_out is not None:
            lp_out[:S].copy_(tp.all_gather(lp, dim=0)[:S])
        self.last_tok[samp["row_slots"][:S].long()] = tok_out[:S]
        self.sampling_dp_steps += 1

    # ------------------------------------------------------------------ graphs
    def capture_graphs(self):
        if not self.use_graphs:
            return
        m = self.model
        torch.cuda.synchronize(self.device)
        pool = torch.cuda.graph_pool_handle()
        stream = torch.cuda.Stream(self.device)
        for b in sorted(self.graph_buckets, reverse=True):
            lay = Layout(b, b, b, b, self.max_blocks)
            buf = torch.zeros(lay.total, dtype=torch.int32, device=self.device)
            G = max(1, m.Hq // m.Hkv)
            w = ops.build_work(np.ones(b, dtype=np.int64), np.full(b, self.max_model_len), G, m.Hkv,
                               self.num_sms, max_splits=m.attn_splits_max, head_dim=m.D)
            # valid dummy metadata for the warm-up / capture runs
            h = torch.zeros(lay.total, dtype=torch.int32)
            o = lay.off
            h[o["qstart"][0]:o["qstart"][0] + b + 1] = torch.arange(b + 1, dtype=torch.int32)
            h[o["seqlen"][0]:o["seqlen"][0] + b] = 1
            h[o["slot"][0]:o["slot"][0] + b] = -1
            h[o["lidx"][0]:o["lidx"][0] + b] = torch.arange(b, dtype=torch.int32)
            h[o["work"][0]:o["work"][0] + 2 * b] = torch.from_numpy(w.work.reshape(-1))
            h[o["topp"][0]:o["topp"][0] + b] = torch.tensor([1.0] * b).view(torch.int32)
            h[o["rslot"][0]:o["rslot"][0] + b] = self.pad_slot
            h[o["sslot"][0]:o["sslot"][0] + b] = self.pad_slot
            h[o["nsplit"][0]] = w.num_splits
            buf.copy_(h)
            fb, samp = self._views(buf, lay, b, b, b, True, w.num_splits)
            tok = torch.zeros(b, dtype=torch.int32, device=self.device)
            lp = torch.zeros(b, dtype=torch.float32, device=self.device)
            stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(stream):
                for _ in range(2):
                    self._forward_and_sample(fb, samp, b, tok, lp)
            torch.cuda.current_stream(self.device).wait_stream(stream)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            n0 = ops._ext.ext().launch_count()
            with torch.cuda.graph(g, pool=pool, stream=stream):
                self._forward_and_sample(fb, samp, b, tok, lp)
            self.graph_kernels[b] = ops._ext.ext().launch_count() - n0
            torch.cuda.synchronize(self.device)
            self.graphs[b] = (g, lay, buf, tok, lp, w.num_splits)

    def _encode_cached(self, mm):
        """Vision encoder output of a request, reused across requests with the same pixels and
        grids (key: content hash) from a bounded LRU cache on the device.  Reference:
        EncoderCacheBlocks (vllm_neuron/vllm/worker/encoder_cache_blocks.py:45-448, slots keyed by
        mm_hash)."""
        import hashlib
        from collections import OrderedDict

        if not hasattr(self, "encoder_cache"):
            self.encoder_cache = OrderedDict()
            self.encoder_cache_hits = 0
        key = hashlib.sha1(mm.pixels.float().contiguous().numpy().tobytes()
                           + repr(mm.grids).encode()).hexdigest()
        hit = self.encoder_cache.get(key)
        if hit is not None:
            self.encoder_cache.move_to_end(key)
            self.encoder_cache_hits += 1
            return hit
        out = self.model.encode_images(mm.pixels.to(self.device), mm.grids)
        self.encoder_cache[key] = out
        while len(self.encoder_cache) > self.encoder_cache_size:
            self.encoder_cache.popitem(last=False)
        return out

    def dummy_forward(self):
        """A one-token forward on the null block that writes no KV and samples nothing: an idle
        data-parallel replica runs it so the collectives inside the model (the MoE all-to-alls
        of wide expert parallelism) stay matched across replicas (reference: the DP dummy batch,
        vllm_neuron/vllm/worker/neuron_model_runner.py:7710)."""
        m = self.model
        lay = Layout(1, 1, 1, 1, self.max_blocks)
        G = self._group()
        w = ops.build_work(np.ones(1, dtype=np.int64), np.ones(1, dtype=np.int64), G, m.Hkv,
                           self.num_sms, max_splits=1, head_dim=m.D)
        h = torch.zeros(lay.total, dtype=torch.int32)
        o = lay.off
        h[o["qstart"][0]:o["qstart"][0] + 2] = torch.arange(2, dtype=torch.int32)
        h[o["seqlen"][0]] = 1
        h[o["lseqlen"][0]] = 1 if self.dcp_rank == 0 else 0
        h[o["slot"][0]] = -1
        h[o["work"][0]:o["work"][0] + 2 * len(w.work)] = torch.from_numpy(w.work.reshape(-1))
        h[o["topp"][0]] = torch.tensor([1.0]).view(torch.int32)
        h[o["rslot"][0]] = self.pad_slot
        h[o["sslot"][0]] = self.pad_slot
        h[o["nsplit"][0]] = w.num_splits
        buf = self.dev_buf[:lay.total]
        buf.copy_(h)
        fb, _ = self._views(buf, lay, 1, 1, len(w.work), True, w.num_splits)
        fb.work = fb.work[:len(w.work)]
        self.model.forward(fb)
        if self.is_cuda:
            torch.cuda.synchronize(self.device)

    def release_graphs(self):
        self.graphs.clear()

    # ------------------------------------------------------------------ execute
    def launch(self, out: SchedulerOutput, want_logprobs: bool = False,
               bitmask: torch.Tensor | None = None, want_ranks: bool = False) -> "StepHandle":
        """Enqueue one step (inputs H2D, forward, sampling, tokens D2H) without waiting."""
        B = len(out.scheduled)
        if B == 0:
            return StepHandle(None, None, None, 0)
        if out.num_tokens > self.max_tokens:
            raise ValueError(f"batch of {out.num_tokens} tokens exceeds max_num_batched_tokens")
        S = sum(s.num_logits for s in out.scheduled)
        self._buf_idx ^= 1
        self.host_buf = self.host_bufs[self._buf_idx]
        self.host_np = self.host_buf.numpy()
        tok_host, lp_host = self.tok_hosts[self._buf_idx], self.lp_hosts[self._buf_idx]
        bucket = None
        if self.use_graphs and out.is_pure_decode and self.graphs and bitmask is None and not want_ranks:
            for bb in sorted(self.graphs):
                if bb >= B:
                    bucket = bb
                    break
        if bucket is not None:
            g, lay, buf, tok, lp, splits = self.graphs[bucket]
            self._pack(out, lay, pad_B=bucket)
            if self.snapshot_dir:
                self._snapshot(out, lay, True, splits)
            n = lay.total
            buf.copy_(self.host_buf[:n], non_blocking=True)
            self.h2d_bytes += n * 4
            g.replay()
            self.num_graph_replays += 1
            self.replayed_kernels += self.graph_kernels.get(bucket, 0)
            tok_src, lp_src = tok, lp
        else:
            lay = Layout(out.num_tokens, B, S, self._max_work_for(out), self.max_blocks)
            S2, decode, splits = self._pack(out, lay)
            W = self._last_work_len
            if self.snapshot_dir:
                self._snapshot(out, lay, decode, splits)
            n = lay.total
            dev = self.dev_buf[:n]
            dev.copy_(self.host_buf[:n], non_blocking=self.is_cuda)
            self.h2d_bytes += n * 4
            fb, samp = self._views(dev, lay, B, S, W, decode, splits)
            fb.work = fb.work[:W]
            fb.prefill_rows = self._last_prefill_rows
            self._attach_prompt_embeds(out, fb)
            self._begin_capture(out)
            if S > 0:
                mask = bitmask.to(self.device, non_blocking=True) if bitmask is not None else None
                self._forward_and_sample(fb, samp, S, self.tok_dev, self.lp_dev, mask,
                                         self.rank_dev if want_ranks else None)
            else:
                self.model.forward(fb)
            self.num_eager_steps += 1
            tok_src, lp_src = self.tok_dev, self.lp_dev
        if S == 0:
            return StepHandle(None, None, None, 0)
        tok_host[:S].copy_(tok_src[:S], non_blocking=self.is_cuda)
        self.d2h_bytes += S * 4
        lps = None
        if want_logprobs:
            lp_host[:S].copy_(lp_src[:S], non_blocking=self.is_cuda)
            self.d2h_bytes += S * 4
            lps = lp_host
        ranks = None
        if want_ranks:
            ranks = self.rank_hosts[self._buf_idx]
            ranks[:S].copy_(self.rank_dev[:S], non_blocking=self.is_cuda)
            self.d2h_bytes += S * 4
        ev = None
        if self.is_cuda:
            ev = torch.cuda.Event()
            ev.record()
        h = StepHandle(ev, tok_host, lps, S)
        h.rank_host = ranks
        return h

    @torch.no_grad()
    def forward_logits(self, out: SchedulerOutput, hidden: bool = False) -> torch.Tensor:
        """Run one step eagerly and return the full-vocabulary logits of its sampling rows
        (``[S, V]``, model dtype) instead of sampling (logit validation / accuracy tooling)."""
        B = len(out.scheduled)
        S = sum(s.num_logits for s in out.scheduled)
        self._buf_idx ^= 1
        self.host_buf = self.host_bufs[self._buf_idx]
        self.host_np = self.host_buf.numpy()
        lay = Layout(out.num_tokens, B, S, self._max_work_for(out), self.max_blocks)
        _, decode, splits = self._pack(out, lay)
        W = self._last_work_len
        if self.snapshot_dir:
            self._snapshot(out, lay, decode, splits)
        dev = self.dev_buf[:lay.total]
        dev.copy_(self.host_buf[:lay.total], non_blocking=self.is_cuda)
        fb, _ = self._views(dev, lay, B, S, W, decode, splits)
        fb.work = fb.work[:W]
        fb.prefill_rows = self._last_prefill_rows
        self._attach_prompt_embeds(out, fb)
        fb.want_hidden = hidden
        self._begin_capture(out)
        logits = self.model.forward(fb).clone()
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
        return logits

    def _begin_capture(self, out: SchedulerOutput):
        """Tell the model's capture session (accuracy tooling) which request and positions each
        row of this step holds."""
        cs = getattr(self.model, "capture", None)
        if cs is None:
            return
        from ..accuracy.tensor_capture import RowGroup, prompt_key

        groups, lgroups, row, lrow = [], [], 0, 0
        for s in out.scheduled:
            key = prompt_key(s.req.prompt_token_ids)
            groups.append(RowGroup(s.req.request_id, key, s.start, s.num_tokens, row))
            row += s.num_tokens
            nl = s.num_logits
            if nl:
                lgroups.append(RowGroup(s.req.request_id, key, s.start + s.num_tokens - nl, nl, lrow))
                lrow += nl
        cs.begin(groups, lgroups)

    def execute(self, out: SchedulerOutput, want_logprobs: bool = False) -> tuple[np.ndarray, np.ndarray | None]:
        """Run one step synchronously; returns sampled tokens (and logprobs) in row order."""
        return self.launch(out, want_logprobs).result()

    def _max_work_for(self, out: SchedulerOutput) -> int:
        G = self._group()
        return sum(math.ceil(s.num_tokens * G / ops.attention.PREFILL_ROWS) for s in out.scheduled) + 1


class StepHandle:
    """Result of a launched step; ``result()`` waits for its device->host copy."""

    def __init__(self, event, tok_host, lp_host, n: int):
        self.event, self.tok_host, self.lp_host, self.n = event, tok_host, lp_host, n
        self.rank_host = None

    @property
    def ranks(self) -> np.ndarray | None:
        """1-based ranks of the sampled tokens (launched with ``want_ranks``; after result())."""
        return self.rank_host[:self.n].numpy().copy() if self.rank_host is not None else None

    def result(self) -> tuple[np.ndarray, np.ndarray | None]:
        if self.n == 0:
            return np.zeros(0, dtype=np.int32), None
        if self.event is not None:
            self.event.synchronize()
        toks = self.tok_host[:self.n].numpy().copy()
        lps = self.lp_host[:self.n].numpy().copy() if self.lp_host is not None else None
        return toks, lps
