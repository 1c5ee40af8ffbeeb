"""Offline inference API: ``LLM(model, ...).generate(prompts, sampling_params)``.

Mirrors the ``vllm.LLM`` call surface the reference's users rely on
(examples/vllm_neuron/models/llama3/run.py: ``LLM(model=..., tensor_parallel_size=...,
additional_config={"neuron_config": {...}})``).  Under ``torchrun`` each rank constructs the
same ``LLM``; tensor parallelism spans the ranks and every rank returns the outputs.
``model`` is a local HF directory, or a HF ``config.json`` dict (random-init weights).
"""
from __future__ import annotations

import os
from typing import Any, Iterable

import torch

from ..config import vision_tp_of
from ..engine.llm_engine import EngineArgs, LLMEngine, RequestOutput
from ..engine.sampling_params import SamplingParams
from ..parallel import state as ps


class EmbeddingOutput:
    def __init__(self, prompt_token_ids: list[int], embedding: list[float]):
        self.prompt_token_ids = prompt_token_ids
        self.outputs = type("Pooled", (), {"embedding": embedding, "data": embedding})()
        self.embedding = embedding


def _normalize_prompt(p: Any, tokenizer) -> list[int]:
    if isinstance(p, dict):
        if "prompt_token_ids" in p:
            return list(p["prompt_token_ids"])
        if "prompt" in p:
            p = p["prompt"]
    if hasattr(p, "prompt_token_ids"):
        return list(p.prompt_token_ids)
    if isinstance(p, str):
        if tokenizer is None:
            raise ValueError("text prompts need a tokenizer; pass token ids or a model dir with one")
        return list(tokenizer.encode(p))
    if isinstance(p, torch.Tensor):
        return p.tolist()
    return [int(x) for x in p]


def _b200_opts(additional_config: dict | None) -> dict:
    a = additional_config or {}
    return a.get("neuron_config") or a.get("b200_config") or {}


class LLM:
    def __init__(self, model, tensor_parallel_size: int = 1, max_num_seqs: int = 256,
                 max_model_len: int | None = None, max_num_batched_tokens: int = 8192,
                 block_size: int = 16, gpu_memory_utilization: float = 0.9,
                 enable_prefix_caching: bool = False, load_format: str = "auto", seed: int = 0,
                 additional_config: dict | None = None, tokenizer: str | None = None,
                 skip_tokenizer_init: bool = False, num_gpu_blocks: int | None = None,
                 enforce_eager: bool = False, device: str | None = None, dtype: str = "auto",
                 async_scheduling: bool | None = None, speculative_config: dict | None = None,
                 data_parallel_size: int | None = None, mm_processor_kwargs: dict | None = None,
                 kv_cache_dtype: str = "auto", enable_expert_parallel: bool = False,
                 kv_transfer_config: dict | None = None, ec_transfer_config: dict | None = None,
                 decode_context_parallel_size: int = 1, **unused):
        if device is None:
            device = f"cuda:{torch.cuda.current_device()}" if torch.cuda.is_available() else "cpu"
        ps.init_distributed(backend="gloo" if str(device).startswith("cpu") else None)
        world = torch.distributed.get_world_size() if torch.distributed.is_initialized() else 1
        if world % tensor_parallel_size:
            raise ValueError(f"tensor_parallel_size={tensor_parallel_size} does not divide the {world} launched ranks")
        dp = world // tensor_parallel_size
        if data_parallel_size not in (None, dp):
            raise ValueError(f"data_parallel_size={data_parallel_size} but TP={tensor_parallel_size} x "
                             f"{world} ranks give {dp}")
        opts = _b200_opts(additional_config)
        # component / attention data parallelism: embedding / MLP / LM head / Q-O heads sharded
        # over TP x DP ranks (all replicas), which then step in lockstep
        cdp = {k: int(opts.get(k, 1) or 1) for k in ("embedding_dp_size", "mlp_dp_size", "lm_head_dp_size",
                                                      "attention_dp_size")}
        for k, v in cdp.items():
            if v > 1 and dp % v:
                raise ValueError(f"{k}={v} must divide the data-parallel size ({dp})")
        st = ps.initialize_parallel_state(ps.ParallelConfig(world_size=world,
                                                            tensor_parallel_size=tensor_parallel_size,
                                                            data_parallel_size=dp,
                                                            decode_context_parallel_size=decode_context_parallel_size,
                                                            component_dp_sizes=tuple(v for v in cdp.values() if v > 1),
                                                            vision_tp_size=vision_tp_of(additional_config)))
        # Data parallelism: each group of TP ranks is an independent engine replica serving
        # every dp-th request; outputs are gathered over the DP group (reference: data
        # parallel replicas, docs/design/parallelism/data_parallelism.md).
        self.dp_size = dp
        self.dp_rank = (torch.distributed.get_rank() // tensor_parallel_size) if world > 1 else 0
        self._ec = None
        if ec_transfer_config is not None:
            # encoder disaggregation: this rank is an encoder instance or a prefill/decode
            # instance receiving vision embeddings (reference: EPD, the EC connector)
            from ..kv_transfer import ECTransferConfig, TensorChannel

            ecc = ECTransferConfig.coerce(ec_transfer_config)
            self._ec = (ecc, TensorChannel(ecc.ec_peer_rank, meta_group=st.cpu))
        if kv_transfer_config is not None or ec_transfer_config is not None:
            # disaggregated prefill / decode: each rank is its own engine (a prefill or a decode
            # instance); the world only carries the KV hand-off
            if tensor_parallel_size != 1:
                raise NotImplementedError("KV transfer engines run with tensor_parallel_size=1")
            self.dp_size, self.dp_rank = 1, 0
        self._dp_group = st.dp_cpu
        # Wide expert parallelism: with data-parallel replicas, an all-to-all backend and
        # enable_expert_parallel, MoE experts are sharded over every rank and tokens move by
        # all-to-all (reference: all2all_backend, vllm_neuron/parallel/all2all.py:33-641).
        nc = (additional_config or {}).get("neuron_config") or (additional_config or {}).get("b200_config") or {}
        st.ep_all2all = bool(dp > 1 and enable_expert_parallel and nc.get("all2all_backend"))
        if dtype == "auto":
            dtype = "bfloat16" if str(device).startswith("cuda") else "float32"
        args = EngineArgs(model=model, max_num_seqs=max_num_seqs,
                          max_num_batched_tokens=max_num_batched_tokens, max_model_len=max_model_len,
                          block_size=block_size, gpu_memory_utilization=gpu_memory_utilization,
                          num_gpu_blocks=num_gpu_blocks, enable_prefix_caching=enable_prefix_caching,
                          load_format=load_format, seed=seed, dtype=dtype, device=device,
                          cuda_graphs=not enforce_eager, async_scheduling=async_scheduling,
                          additional_config=additional_config or {},
                          speculative_config=speculative_config, kv_cache_dtype=kv_cache_dtype,
                          kv_transfer_config=kv_transfer_config,
                          decode_context_parallel_size=decode_context_parallel_size)
        self.engine = LLMEngine(args, tp=st.tp)
        self.mm_processor_kwargs = mm_processor_kwargs
        self.tokenizer = None
        if not skip_tokenizer_init:
            path = tokenizer or (model if isinstance(model, str) else None)
            if path and any(os.path.exists(os.path.join(path, f)) for f in
                            ("tokenizer.json", "tokenizer.model", "tokenizer_config.json")):
                from transformers import AutoTokenizer

                self.tokenizer = AutoTokenizer.from_pretrained(path)
        self.engine.tokenizer = self.tokenizer

    def get_tokenizer(self):
        return self.tokenizer

    def generate(self, prompts, sampling_params: SamplingParams | list | None = None,
                 use_tqdm: bool = False) -> list[RequestOutput]:
        if isinstance(prompts, (str, dict)) or (isinstance(prompts, list) and prompts and isinstance(prompts[0], int)):
            prompts = [prompts]
        prompts = list(prompts)
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(prompts)
        if self.dp_size > 1:
            return self._generate_dp(prompts, sampling_params)
        return self._generate(prompts, sampling_params)

    def _generate_dp(self, prompts, sampling_params) -> list[RequestOutput]:
        mine = [i for i in range(len(prompts)) if i % self.dp_size == self.dp_rank]
        if getattr(self.engine.model, "a2a", None) is not None or getattr(self.engine.model, "dpcol", None) is not None:
            # replicas share the MoE layers' all-to-alls: step in lockstep, idle ones run a
            # one-token dummy forward (reference: DP dummy batch, neuron_model_runner.py:7710)
            local = self._generate([prompts[i] for i in mine], [sampling_params[i] for i in mine],
                                   lockstep=self._dp_group)
        else:
            local = self._generate([prompts[i] for i in mine], [sampling_params[i] for i in mine]) if mine else []
        parts = [None] * self.dp_size
        torch.distributed.all_gather_object(parts, (mine, local), group=self._dp_group)
        res = [None] * len(prompts)
        for idx, outs in parts:
            for i, o in zip(idx, outs):
                res[i] = o
        return res

    # ------------------------------------------------------------ encoder disaggregation
    @staticmethod
    def _mm_hash(mm) -> str:
        import hashlib

        return hashlib.sha1(mm.pixels.float().contiguous().numpy().tobytes()).hexdigest()

    @torch.no_grad()
    def encode_remote(self, prompts) -> int:
        """Encoder instance: run the vision encoder of every image prompt and send the merged
        embeddings (and DeepStack features) to the prefill/decode instance, in prompt order.
        Returns the number of encodings sent."""
        from ..engine.multimodal import prepare_image_request

        if self._ec is None or self._ec[0].ec_role != "ec_producer":
            raise RuntimeError("encode_remote needs ec_transfer_config with ec_role='ec_producer'")
        sent = 0
        dev = self.engine.device
        for p in prompts:
            if not (isinstance(p, dict) and p.get("multi_modal_data")):
                continue
            toks = _normalize_prompt(p, self.tokenizer)
            _, mm = prepare_image_request(toks, p["multi_modal_data"].get("image"), self.engine.model,
                                          self.engine.model_path, self.mm_processor_kwargs)
            emb, deep = self.engine.model.encode_images(mm.pixels.to(dev), mm.grids)
            deep = deep if deep is not None else torch.zeros(0, dtype=emb.dtype, device=dev)
            self._ec[1].send({"mm_hash": self._mm_hash(mm)}, [emb, deep])
            sent += 1
        return sent

    def _install_remote_encoding(self, mm):
        meta, (emb, deep) = self._ec[1].recv(self.engine.device)
        if meta["mm_hash"] != self._mm_hash(mm):
            raise RuntimeError("received vision embeddings for a different image (requests out of order)")
        mm.emb = emb
        mm.deep = deep if deep.numel() else None

    def generate_remote(self, num_requests: int, sampling_params=None) -> list[RequestOutput]:
        """Decode engine of a disaggregated pair: receive ``num_requests`` requests (prompt, the
        prefill engine's tokens and their KV) and decode them to completion.
        ``sampling_params``: one SamplingParams for all, or a dict / callable from request id
        (a routing proxy knows each request's decode parameters).  Outputs are in arrival order
        and include the tokens the prefill engine sampled."""
        if self.engine.kv_connector is None or not self.engine.kv_transfer.is_consumer:
            raise RuntimeError("generate_remote needs kv_transfer_config with kv_role='kv_consumer'")
        reqs = [self.engine.recv_remote(sampling_params) for _ in range(num_requests)]
        done = {r.request_id: r for r in reqs if r.status.finished}
        for r in self.engine.run_until_done():
            done[r.request_id] = r
        outs = []
        for r in reqs:
            o = LLMEngine.to_output(done[r.request_id])
            if self.tokenizer is not None:
                for c in o.outputs:
                    c.text = self.tokenizer.decode(c.token_ids, skip_special_tokens=True)
            outs.append(o)
        return outs

    def _generate(self, prompts, sampling_params, lockstep=None) -> list[RequestOutput]:
        ids = []
        base = self.engine.num_steps * 1_000_003
        for i, (p, sp) in enumerate(zip(prompts, sampling_params)):
            if isinstance(p, dict) and "prompt_embeds" in p:
                emb = p["prompt_embeds"]
                ids.append(self.engine.add_request([0] * emb.shape[0], sp, request_id=f"gen-{base}-{i}",
                                                   prompt_embeds=emb))
                continue
            if isinstance(p, dict) and p.get("multi_modal_data"):
                from ..engine.multimodal import prepare_image_request

                toks = _normalize_prompt(p, self.tokenizer)
                images = p["multi_modal_data"].get("image")
                if p["multi_modal_data"].get("video") is not None:
                    from ..engine.multimodal import prepare_video_request

                    toks, mm = prepare_video_request(toks, p["multi_modal_data"]["video"], self.engine.model,
                                                     self.engine.model_path, self.mm_processor_kwargs,
                                                     fps=float(p.get("fps", 2.0)), images=images)
                else:
                    toks, mm = prepare_image_request(toks, images, self.engine.model, self.engine.model_path,
                                                     self.mm_processor_kwargs)
                if self._ec is not None and self._ec[0].ec_role == "ec_consumer":
                    self._install_remote_encoding(mm)
                ids.append(self.engine.add_request(toks, sp, request_id=f"gen-{base}-{i}", mm=mm))
                continue
            toks = _normalize_prompt(p, self.tokenizer)
            ids.append(self.engine.add_request(toks, sp, request_id=f"gen-{base}-{i}"))
        done = {r.request_id: r for r in (self.engine.run_lockstep(lockstep) if lockstep is not None
                                          else self.engine.run_until_done())}
        outs = []
        for rid in ids:
            o = LLMEngine.to_output(done[rid])
            if self.tokenizer is not None:
                for c in o.outputs:
                    c.text = self.tokenizer.decode(c.token_ids, skip_special_tokens=True)
            outs.append(o)
        return outs

    def embed(self, prompts, normalize: bool = True, batch_size: int | None = None) -> list["EmbeddingOutput"]:
        """Pooling API (embedding models such as Qwen3-Embedding): last-token pooling of the
        final hidden state, L2-normalised (reference: the runner's ``_pool``, LAST + normalize,
        vllm_neuron/vllm/worker/neuron_model_runner.py:7984 and model/pooling_adapter.py)."""
        if isinstance(prompts, (str, dict)) or (isinstance(prompts, list) and prompts and isinstance(prompts[0], int)):
            prompts = [prompts]
        toks = [_normalize_prompt(p, self.tokenizer) for p in prompts]
        bs = batch_size or self.engine.args.max_num_seqs
        outs = []
        for i in range(0, len(toks), bs):
            h = self.engine.prompt_hidden(toks[i:i + bs])
            if normalize:
                h = torch.nn.functional.normalize(h, dim=-1)
            outs += [EmbeddingOutput(t, e.tolist()) for t, e in zip(toks[i:i + bs], h)]
        return outs

    encode = embed

    def shutdown(self):
        self.engine.shutdown()
