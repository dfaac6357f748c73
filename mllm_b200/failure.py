"""Failure detection for the tensor-parallel ranks, on the host.

The reference has one process and catches exceptions per request (Scheduler.cpp:59-75,
QwenRunner.cpp:57-66); it has no peers to lose.  Sharding attention over GPUs makes every layer
wait on every rank, so a rank that dies or leaves must be noticed before the others launch a
collective that can never complete.  Two mechanisms cover that:

* `PeerMonitor` -- a heartbeat in the process group's key-value store.  A thread bumps this
  rank's counter every `interval` seconds; `check()` (called between steps, before the next
  launch) raises `PeerLost` when a peer has said it is leaving, or when its counter has not
  moved for `timeout` seconds, or when the store itself is gone (its host rank died).  The
  caller then aborts its communicators (`mllm_comm_abort`) instead of launching.
* the communicators' own watchdog (mllm_comm_*, include/mllm_attn.h): a collective still
  running after its deadline, or an asynchronous NCCL error, aborts the communicator, and every
  later call reports MLLM_ERR_COMM / MLLM_ERR_COMM_TIMEOUT.

Nothing here touches a GPU: a rank leaves only between steps, with none of its work in flight.
"""
from __future__ import annotations

import threading
import time


class PeerLost(RuntimeError):
    """A peer rank has left, died or stopped beating."""

    def __init__(self, rank: int, why: str):
        self.rank = rank
        super().__init__(f"peer rank {rank} lost: {why}")


class PeerMonitor:
    """Heartbeats of `world` ranks through a torch.distributed Store (TCPStore, FileStore...).

    Every rank constructs one (collectively: construction waits, up to `timeout`, for every
    peer's first beat) and calls `check()` between steps.  `leave()` tells the peers this rank
    is going away on purpose; `close()` stops this rank's beat."""

    def __init__(self, store, rank: int, world: int, interval: float = 0.05, timeout: float = 1.0,
                 prefix: str = "mllm_hb"):
        if not 0 <= rank < world:
            raise ValueError("PeerMonitor: rank out of range")
        if not 0 < interval < timeout:
            raise ValueError("PeerMonitor: need 0 < interval < timeout")
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._count = 0
        self._seen = {}          # peer -> (last counter, host time it last changed)
        self._stop = threading.Event()
        self._beat()
        self._thread = threading.Thread(target=self._run, name=f"mllm-heartbeat-{rank}", daemon=True)
        self._thread.start()
        deadline = time.monotonic() + timeout
        for p in self.peers():
            while True:
                try:
                    if self.store.check([self._key("beat", p)]):
                        break
                except Exception as e:   # the store's host is gone
                    raise PeerLost(p, f"store unreachable ({e})") from e
                if time.monotonic() > deadline:
                    raise PeerLost(p, "no first heartbeat")
                time.sleep(interval / 4)
            self._seen[p] = (None, time.monotonic())

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def peers(self):
        return [p for p in range(self.world) if p != self.rank]

    def _beat(self):
        self._count += 1
        self.store.set(self._key("beat", self.rank), str(self._count))

    def _run(self):
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:
                return   # the store is gone; check() reports it

    def check(self) -> None:
        """Raises PeerLost if any peer left, died or went silent for longer than `timeout`."""
        now = time.monotonic()
        for p in self.peers():
            try:
                if self.store.check([self._key("left", p)]):
                    raise PeerLost(p, "left")
                val = self.store.get(self._key("beat", p))
            except PeerLost:
                raise
            except Exception as e:
                raise PeerLost(p, f"store unreachable ({e})") from e
            last, since = self._seen[p]
            if val != last:
                self._seen[p] = (val, now)
            elif now - since > self.timeout:
                raise PeerLost(p, f"no heartbeat for {now - since:.2f} s")

    def leave(self) -> None:
        """Tells the peers that this rank is leaving (between steps), then stops beating."""
        try:
            self.store.set(self._key("left", self.rank), "1")
        finally:
            self.close()

    def close(self) -> None:
        self._stop.set()
        if self._thread.is_alive() and self._thread is not threading.current_thread():
            self._thread.join(timeout=5 * self.interval + 1.0)
