"""Host-side failure detection for multi-rank serving.

Every rank publishes a heartbeat (its wall-clock time) under ``hb/<rank>`` in a
``torch.distributed`` key-value store from a daemon thread; :meth:`PeerMonitor.check` reads the
peers' entries before a step is launched and raises :class:`PeerFailureError` when a peer has
announced its exit (``exit/<rank>``) or its heartbeat is older than the timeout.  A rank therefore
learns that a peer is gone on the host, between steps, before it launches a kernel or collective
that would wait for that peer (the device-side waits of the fused collectives are bounded as a
second line of defence and report through the status word).

Reference counterparts: the gloo barrier timeouts (``VLLM_NEURON_BARRIER_TIMEOUT``,
parallel/neuron_parallel_state.py:1568-1604) and the NIXL heartbeats
(vllm/kv_connector/neuron_nixl_connector.py:363-398).
"""
from __future__ import annotations

import datetime
import threading
import time

import torch.distributed as dist

from ..exceptions import B200Error


class PeerFailureError(B200Error):
    """A peer rank exited or stopped sending heartbeats."""

    def __init__(self, rank: int, why: str):
        self.rank = rank
        super().__init__(f"peer rank {rank} failed: {why}")


class PeerMonitor:
    def __init__(self, store: dist.Store, rank: int, world: int, interval_s: float = 0.5,
                 timeout_s: float = 10.0, prefix: str = "b200"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout = interval_s, timeout_s
        self.prefix = prefix
        self._stop = threading.Event()
        self._beat()
        self._thread = threading.Thread(target=self._run, name=f"b200-heartbeat-{rank}", daemon=True)
        self._thread.start()
        # every peer has published once before anyone checks (start-up is not a failure)
        peers = [self._key("hb", r) for r in range(world) if r != rank]
        if peers:
            try:
                store.wait(peers, datetime.timedelta(seconds=max(timeout_s, 30.0)))
            except Exception as e:
                raise PeerFailureError(-1, f"peers did not start within {max(timeout_s, 30.0)} s: {e}")

    def _key(self, kind: str, r: int) -> str:
        return f"{self.prefix}/{kind}/{r}"

    def _beat(self):
        self.store.set(self._key("hb", self.rank), repr(time.time()))

    def _run(self):
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:  # store gone: the process is shutting down
                return

    def stop(self, announce_exit: bool = True):
        """Stop beating; with ``announce_exit`` the peers learn at once that this rank left."""
        self._stop.set()
        self._thread.join(timeout=5)
        if announce_exit:
            try:
                self.store.set(self._key("exit", self.rank), "1")
                self.store.add(f"{self.prefix}/exits", 1)
            except Exception:
                pass

    def check_fast(self):
        """One store round trip: raise if any peer announced its exit (run before every step)."""
        if self.store.add(f"{self.prefix}/exits", 0) > 0:
            self.check()

    def check(self):
        """Raise :class:`PeerFailureError` for the first peer that exited or went silent."""
        now = time.time()
        for r in range(self.world):
            if r == self.rank:
                continue
            if self.store.check([self._key("exit", r)]):
                raise PeerFailureError(r, "announced exit")
            if not self.store.check([self._key("hb", r)]):
                raise PeerFailureError(r, "no heartbeat published")
            last = float(self.store.get(self._key("hb", r)).decode())
            if now - last > self.timeout:
                raise PeerFailureError(r, f"last heartbeat {now - last:.1f} s ago (timeout {self.timeout} s)")


def make_store(host: str, port: int, rank: int, world: int, timeout_s: float = 30.0) -> dist.TCPStore:
    """A TCP store for the heartbeats, separate from the process group's own store."""
    return dist.TCPStore(host, port, world, rank == 0, timeout=datetime.timedelta(seconds=timeout_s),
                         wait_for_workers=False)
