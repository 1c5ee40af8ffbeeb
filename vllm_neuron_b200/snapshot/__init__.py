"""Runtime input snapshots: capture the packed device inputs of selected engine steps (with a
JSON metadata record per step) and replay a captured step through a runner.

* :mod:`.config` -- which steps to capture (step index, token position, request id, rank) and
  where, from ``VLLM_B200_SNAPSHOT_*`` variables;
* :mod:`.capture` -- :class:`SnapshotCapturer`, called by the model runner before each step;
* :mod:`.meta` -- the per-step metadata record;
* :mod:`.replay` -- load a snapshot and run it again (prefill steps with no cached context
  reproduce their logits exactly; decode steps need the KV cache they ran against).

Reference: vllm_neuron/snapshot/ (config.py selection rules, capture.py, context.py, meta.py).
"""
from .capture import SnapshotCapturer
from .config import CaptureSelector, SnapshotConfig
from .replay import load_snapshot, replay_logits

__all__ = ["SnapshotCapturer", "CaptureSelector", "SnapshotConfig", "load_snapshot", "replay_logits"]
