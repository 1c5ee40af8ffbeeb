"""KV-cache transfer between a prefill engine (producer) and a decode engine (consumer).

A producer engine runs the prompt (prefill plus the first sampled token) of each request and
then hands the request over: its metadata (request id, prompt tokens, sampled tokens) and the
KV of every token but the last, gathered from the paged cache block by block for every layer
into one tensor ``[layers, 2, blocks, kv_heads, block_size, head_dim]``.  The consumer
allocates blocks in its own cache, scatters the KV into them and continues the request as a
running decode from the last sampled token.

Transport: ``torch.distributed`` point-to-point between the two engine processes (ranks of one
world): metadata through the gloo group, the KV tensor through the default group (NCCL over
NVLink between two GPUs of a node; gloo on CPU).  Cross-node RDMA (the reference's NIXL
transport) is out of scope.

Reference: ``NeuronNixlConnector`` (vllm_neuron/vllm/kv_connector/neuron_nixl_connector.py:
59-819) and docs/design/vllm/disaggregated-inference.md (a prefill node and a decode node, the
prompt's KV moved per request, the decode node continuing from the first token).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class KVTransferConfig:
    kv_role: str = "kv_producer"      # "kv_producer" (prefill) or "kv_consumer" (decode)
    kv_connector: str = "TorchDistConnector"
    kv_peer_rank: int = -1            # world rank of the other engine (-1: the other of two)

    @classmethod
    def coerce(cls, c) -> "KVTransferConfig | None":
        if c is None or isinstance(c, cls):
            return c
        c = dict(c)
        cfg = cls(**{k: v for k, v in c.items() if k in ("kv_role", "kv_connector", "kv_peer_rank")})
        if cfg.kv_role not in ("kv_producer", "kv_consumer"):
            raise ValueError(f"kv_role must be kv_producer or kv_consumer, got {cfg.kv_role!r}")
        if cfg.kv_connector not in ("TorchDistConnector", "NixlConnector", "NeuronNixlConnector"):
            raise ValueError(f"unknown kv_connector {cfg.kv_connector!r}")
        return cfg

    @property
    def is_producer(self) -> bool:
        return self.kv_role == "kv_producer"

    @property
    def is_consumer(self) -> bool:
        return self.kv_role == "kv_consumer"


class TorchDistKVConnector:
    def __init__(self, config: KVTransferConfig, meta_group=None, data_group=None):
        if not dist.is_initialized():
            raise RuntimeError("KV transfer needs torch.distributed (one rank per engine)")
        self.cfg = config
        self.peer = config.kv_peer_rank if config.kv_peer_rank >= 0 else 1 - dist.get_rank()
        self.meta_group = meta_group
        self.data_group = data_group
        self.sent = 0
        self.received = 0
        self.bytes = 0

    @staticmethod
    def gather_kv(kv_caches, block_ids: list[int]) -> torch.Tensor:
        """``[layers, 2, blocks, kv_heads, block_size, head_dim]`` of the given blocks."""
        idx = torch.tensor(block_ids, dtype=torch.long, device=kv_caches[0][0].device)
        return torch.stack([torch.stack([k.index_select(0, idx), v.index_select(0, idx)])
                            for k, v in kv_caches])

    @staticmethod
    def scatter_kv(kv_caches, block_ids: list[int], kv: torch.Tensor) -> None:
        idx = torch.tensor(block_ids, dtype=torch.long, device=kv_caches[0][0].device)
        for l, (k, v) in enumerate(kv_caches):
            k.index_copy_(0, idx, kv[l, 0].to(k.dtype))
            v.index_copy_(0, idx, kv[l, 1].to(v.dtype))

    def send_request(self, meta: dict, kv: torch.Tensor) -> None:
        meta = dict(meta, kv_shape=list(kv.shape), kv_dtype=str(kv.dtype).replace("torch.", ""))
        dist.send_object_list([meta], dst=self.peer, group=self.meta_group)
        if kv.numel():
            payload = kv.contiguous()
            if payload.dtype == torch.float8_e4m3fn:  # sent as raw bytes
                payload = payload.view(torch.uint8)
            dist.send(payload, dst=self.peer, group=self.data_group)
            self.bytes += payload.numel() * payload.element_size()
        self.sent += 1

    def recv_request(self, device: torch.device) -> tuple[dict, torch.Tensor]:
        box = [None]
        dist.recv_object_list(box, src=self.peer, group=self.meta_group)
        meta = box[0]
        dtype = getattr(torch, meta["kv_dtype"])
        wire = torch.uint8 if dtype == torch.float8_e4m3fn else dtype
        kv = torch.empty(meta["kv_shape"], dtype=wire, device=device)
        if kv.numel():
            dist.recv(kv, src=self.peer, group=self.data_group)
            self.bytes += kv.numel() * kv.element_size()
        if wire != dtype:
            kv = kv.view(dtype)
        self.received += 1
        return meta, kv


@dataclass
class ECTransferConfig:
    """Encoder disaggregation: an encoder instance (``ec_producer``) runs the vision encoder of
    image requests and sends the embeddings to a prefill/decode instance (``ec_consumer``)."""

    ec_role: str = "ec_producer"
    ec_peer_rank: int = -1

    @classmethod
    def coerce(cls, c) -> "ECTransferConfig | None":
        if c is None or isinstance(c, cls):
            return c
        cfg = cls(**{k: v for k, v in dict(c).items() if k in ("ec_role", "ec_peer_rank")})
        if cfg.ec_role not in ("ec_producer", "ec_consumer"):
            raise ValueError(f"ec_role must be ec_producer or ec_consumer, got {cfg.ec_role!r}")
        return cfg


class TensorChannel:
    """Point-to-point channel of (metadata, tensors) messages between two engine processes:
    metadata through a gloo group, tensors through ``data_group`` (NCCL between GPUs, gloo on
    CPU).  Reference: the EC connector (vllm_neuron/vllm/ec_connector/neuron_nixl_ec_connector.py)
    moving encoder outputs between instances."""

    def __init__(self, peer: int = -1, meta_group=None, data_group=None):
        self.peer = peer if peer >= 0 else 1 - dist.get_rank()
        self.meta_group = meta_group
        self.data_group = data_group

    def send(self, meta: dict, tensors: list[torch.Tensor]) -> None:
        specs = [(list(t.shape), str(t.dtype).replace("torch.", "")) for t in tensors]
        dist.send_object_list([dict(meta, _tensors=specs)], dst=self.peer, group=self.meta_group)
        for t in tensors:
            if t.numel():
                dist.send(t.contiguous(), dst=self.peer, group=self.data_group)

    def recv(self, device) -> tuple[dict, list[torch.Tensor]]:
        box = [None]
        dist.recv_object_list(box, src=self.peer, group=self.meta_group)
        meta = box[0]
        out = []
        for shape, dt in meta.pop("_tensors"):
            t = torch.empty(shape, dtype=getattr(torch, dt), device=device)
            if t.numel():
                dist.recv(t, src=self.peer, group=self.data_group)
            out.append(t)
        return meta, out
