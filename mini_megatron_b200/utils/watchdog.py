"""Rank failure detection between training steps.

The reference relies on NCCL's default timeouts only.  Here every rank runs a
small heartbeat thread that writes ``mmb/hb/<rank>`` (a wall-clock stamp) into
the process group's key-value store and reads the other ranks' stamps.  A
rank whose stamp is older than ``timeout`` seconds -- or that wrote
``mmb/exit/<rank>`` -- is reported as failed.  ``check()`` raises
:class:`RankFailure` on the host, BETWEEN steps, so no collective or kernel is
in flight when a job decides to stop; the process group's own timeout (set
short via ``init_process_group(timeout=...)``) bounds a collective that was
already issued when a peer died.

Failure is detected on the host only: nothing here faults or stalls a GPU.
"""
from __future__ import annotations

import threading
import time

import torch.distributed as dist


class RankFailure(RuntimeError):
    def __init__(self, ranks, reason):
        super().__init__(f"rank(s) {sorted(ranks)} failed: {reason}")
        self.ranks = sorted(ranks)
        self.reason = reason


class Heartbeat:
    PREFIX = "mmb/hb/"
    EXIT = "mmb/exit/"

    def __init__(self, store=None, rank=None, world=None, interval=0.25, timeout=3.0):
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.interval, self.timeout = interval, timeout
        self.failed = {}
        self._stop = threading.Event()
        self._last_seen = {}
        self._thread = threading.Thread(target=self._run, name="mmb-heartbeat", daemon=True)

    def start(self):
        self._beat()
        self._thread.start()
        return self

    def _beat(self):
        self.store.set(f"{self.PREFIX}{self.rank}", repr(time.time()))

    def _run(self):
        start = time.time()
        while not self._stop.wait(self.interval):
            try:
                self._beat()
                now = time.time()
                for r in range(self.world):
                    if r == self.rank or r in self.failed:
                        continue
                    if self.store.check([f"{self.EXIT}{r}"]):
                        self.failed[r] = "announced exit"
                        continue
                    if not self.store.check([f"{self.PREFIX}{r}"]):
                        if now - start > self.timeout:
                            self.failed[r] = "never joined"
                        continue
                    stamp = float(self.store.get(f"{self.PREFIX}{r}").decode())
                    prev = self._last_seen.get(r)
                    if prev is None or stamp != prev[0]:
                        self._last_seen[r] = (stamp, now)
                    elif now - prev[1] > self.timeout:
                        self.failed[r] = f"no heartbeat for {now - prev[1]:.1f}s"
            except Exception as exc:  # noqa: BLE001 -- the store itself went away
                self.failed[-1] = f"store unreachable: {exc}"

    def check(self):
        """Raise RankFailure if any peer was detected as failed."""
        if self.failed:
            raise RankFailure(list(self.failed), "; ".join(f"{r}: {m}" for r, m in self.failed.items()))

    def announce_exit(self):
        """Tell the peers this rank is leaving on purpose (between steps)."""
        self.store.set(f"{self.EXIT}{self.rank}", "1")

    def stop(self):
        self._stop.set()
        self._thread.join(timeout=2 * self.interval + 1)
