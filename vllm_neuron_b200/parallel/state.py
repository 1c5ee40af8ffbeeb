"""Process groups of every parallelism the framework supports, built from pure rank math.

All group layouts are computed by pure functions (unit-tested on CPU) and then instantiated
with ``torch.distributed.new_group`` -- NCCL device groups for tensor traffic plus gloo CPU
groups for control (barriers, DP padding reduce).  Rank order is contiguous: NVSwitch gives
every GPU the same bandwidth to every peer, so the Trn2 mesh/torus helpers of the reference
collapse to the identity.

Reference: vllm_neuron/parallel/neuron_parallel_state.py (group builders :99-701,
init_neuron_distributed_environment :764-844, getters :1177-1460, barriers :1568-1604).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from .comm import GroupComm


# ------------------------------------------------------------------------- rank math
def tp_groups(world: int, tp: int) -> list[list[int]]:
    """Consecutive TP groups: [[0..tp-1], [tp..2tp-1], ...]."""
    assert world % tp == 0
    return [list(range(i, i + tp)) for i in range(0, world, tp)]


def dp_groups(world: int, tp: int) -> list[list[int]]:
    """Ranks with the same TP index across DP replicas."""
    dp = world // tp
    return [[d * tp + t for d in range(dp)] for t in range(tp)]


def ep_groups(world: int, ep: int) -> list[list[int]]:
    """Expert-parallel groups of size ``ep`` (consecutive); ep defaults to TP x DP."""
    assert world % ep == 0
    return [list(range(i, i + ep)) for i in range(0, world, ep)]


def ep_tp_groups(world: int, ep: int) -> list[list[int]]:
    """Ranks that share the same experts (intermediate dim sharded) when ep < world
    (reference ``_build_ep_group_ranks``, neuron_parallel_state.py:99-113)."""
    n = world // ep
    return [[e + k * ep for k in range(n)] for e in range(ep)]


def sub_groups(group: list[int], inner: int) -> tuple[list[list[int]], list[list[int]]]:
    """Split a group into ``inner``-sized contiguous sub-groups (e.g. attention TP inside a
    TP x attn-DP supergroup) and the orthogonal groups (attention DP)."""
    assert len(group) % inner == 0
    outer = len(group) // inner
    inner_g = [group[i * inner:(i + 1) * inner] for i in range(outer)]
    outer_g = [[group[i * inner + j] for i in range(outer)] for j in range(inner)]
    return inner_g, outer_g


def dcp_groups(tp_group: list[int], dcp: int) -> tuple[list[list[int]], list[list[int]]]:
    """Decode-context-parallel KV groups inside a TP group: ranks ``r, r + tp/dcp, ...`` share
    the KV-head shard and split tokens (reference: neuron_parallel_state.py:393-447)."""
    tp = len(tp_group)
    assert tp % dcp == 0
    stride = tp // dcp
    kv = [[tp_group[s + k * stride] for k in range(dcp)] for s in range(stride)]
    head = [tp_group[i * stride:(i + 1) * stride] for i in range(dcp)]
    return kv, head


def dcp_decode_groups(tp_group: list[int], dcp: int) -> list[list[int]]:
    """Decode-context-parallel replica sets: ``dcp`` consecutive TP ranks, which share their
    (replicated) KV heads when TP exceeds the KV head count, split the tokens of every sequence
    (``dcp_rank = tp_rank % dcp``; reference: docs/design/parallelism/dcp.md, "DCP Decode")."""
    assert len(tp_group) % dcp == 0
    return [tp_group[i:i + dcp] for i in range(0, len(tp_group), dcp)]


@dataclass
class ParallelConfig:
    world_size: int = 1
    tensor_parallel_size: int = 1
    data_parallel_size: int = 1
    expert_parallel_size: int | None = None
    decode_context_parallel_size: int = 1
    attention_dp_size: int = 1
    vision_tp_size: int = 1
    # component / attention DP sizes in use (k replicas share each such component)
    component_dp_sizes: tuple = ()

    @property
    def component_dp(self) -> bool:
        return bool(self.component_dp_sizes)

    def validate(self):
        if self.tensor_parallel_size * self.data_parallel_size != self.world_size:
            raise ValueError("world_size must equal TP x DP")
        if self.tensor_parallel_size % self.decode_context_parallel_size:
            raise ValueError("DCP size must divide TP")
        if self.tensor_parallel_size % self.vision_tp_size:
            raise ValueError("vision_tp_size must divide TP")
        for k in self.component_dp_sizes:
            if k < 2 or self.data_parallel_size % k:
                raise ValueError(f"a component DP size of {k} must divide the data-parallel size "
                                 f"({self.data_parallel_size})")
        ep = self.expert_parallel_size or self.world_size
        if self.world_size % ep:
            raise ValueError("EP size must divide the world size")


@dataclass
class ParallelState:
    rank: int = 0
    config: ParallelConfig = field(default_factory=ParallelConfig)
    tp: GroupComm = field(default_factory=lambda: GroupComm(None))
    dp: GroupComm = field(default_factory=lambda: GroupComm(None))
    ep: GroupComm = field(default_factory=lambda: GroupComm(None))
    dcp: GroupComm = field(default_factory=lambda: GroupComm(None))
    vision_tp: GroupComm = field(default_factory=lambda: GroupComm(None))
    world: GroupComm = field(default_factory=lambda: GroupComm(None))  # component DP: TP x DP ranks
    # component DP size k -> (DP column of k replicas, TP x k component group) of this rank
    cdp: dict = field(default_factory=dict)
    cpu: dist.ProcessGroup | None = None
    dp_cpu: dist.ProcessGroup | None = None   # gloo group of this rank's DP peers
    groups: dict = field(default_factory=dict)
    # MoE experts sharded over the EP group with all-to-all token exchange (wide EP across
    # data-parallel replicas); replicas then step in lockstep
    ep_all2all: bool = False


_STATE: ParallelState | None = None


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> tuple[int, int]:
    """Initialise torch.distributed from the torchrun environment (no-op for one process)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world == 1 or dist.is_initialized():
        return (dist.get_rank() if dist.is_initialized() else 0,
                dist.get_world_size() if dist.is_initialized() else 1)
    local = int(os.environ.get("LOCAL_RANK", rank))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
    kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(**kw)
    return rank, world


def _make(groups: list[list[int]], rank: int, backend: str | None = None) -> tuple[GroupComm, list[int]]:
    mine = None
    mine_ranks = [rank]
    for g in groups:
        pg = dist.new_group(g, backend=backend) if len(g) > 1 else None
        if rank in g:
            mine, mine_ranks = pg, g
    return GroupComm(mine, mine_ranks), mine_ranks


def initialize_parallel_state(cfg: ParallelConfig) -> ParallelState:
    """Build every group (all ranks must call this with the same config)."""
    global _STATE
    cfg.validate()
    if not dist.is_initialized() or cfg.world_size == 1:
        _STATE = ParallelState(0, cfg)
        return _STATE
    rank = dist.get_rank()
    W, tp = cfg.world_size, cfg.tensor_parallel_size
    st = ParallelState(rank, cfg)
    st.tp, tp_ranks = _make(tp_groups(W, tp), rank)
    st.dp, _ = _make(dp_groups(W, tp), rank)
    st.ep, _ = _make(ep_groups(W, cfg.expert_parallel_size or W), rank)
    if cfg.decode_context_parallel_size > 1:
        sets = []
        for g in tp_groups(W, tp):
            sets.extend(dcp_decode_groups(g, cfg.decode_context_parallel_size))
        st.dcp, _ = _make(sets, rank)
    if cfg.vision_tp_size > 1:  # vision encoder TP: consecutive ranks of each TP group
        sets = []
        for g in tp_groups(W, tp):
            sets.extend(sub_groups(g, cfg.vision_tp_size)[0])
        st.vision_tp, _ = _make(sets, rank)
    for k in sorted(set(cfg.component_dp_sizes)):
        cols, comps = [], []
        for g in range(W // tp // k):  # replicas [g k, (g + 1) k)
            comps.append(list(range(g * k * tp, (g + 1) * k * tp)))
            cols.extend([[(g * k + i) * tp + t for i in range(k)] for t in range(tp)])
        dc, _ = _make(cols, rank)
        cg, _ = _make(comps, rank)
        st.cdp[k] = (dc, cg)
        if k == W // tp:
            st.world = cg
    st.cpu = dist.new_group(list(range(W)), backend="gloo")
    if W // tp > 1:
        for g in dp_groups(W, tp):
            pg = dist.new_group(g, backend="gloo")
            if rank in g:
                st.dp_cpu = pg
    _STATE = st
    return st


def get_parallel_state() -> ParallelState:
    global _STATE
    if _STATE is None:
        _STATE = ParallelState()
    return _STATE


def world_barrier(timeout_s: float | None = None):
    """Barrier over the gloo CPU group with a timeout (reference: world_barrier,
    neuron_parallel_state.py:1568-1604; timeout from VLLM_NEURON_BARRIER_TIMEOUT)."""
    st = get_parallel_state()
    if st.cpu is None:
        return
    from .. import envs

    timeout_s = timeout_s if timeout_s is not None else envs.VLLM_B200_BARRIER_TIMEOUT
    st.cpu.barrier().wait(datetime.timedelta(seconds=timeout_s))


def destroy_parallel_state():
    global _STATE
    _STATE = None
    if dist.is_initialized():
        dist.destroy_process_group()
