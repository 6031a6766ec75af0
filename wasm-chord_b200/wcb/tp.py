"""Failure detection for a tensor-parallel group, on the host.

One process per GPU holds one rank of the model. A rank that stops (its process
exits or hangs) leaves the others waiting for its partial sums: the device-side
waits of the peer exchange end after ``wait_ms`` with an error, and an NCCL
collective would wait for good. ``Watchdog`` lets the ranks learn of a failure
on the host before they launch the next step: every rank publishes a counter
in a shared ``torch.distributed`` store (TCPStore, FileStore, ...) every
``interval`` seconds, and a rank whose counter has not moved for ``timeout``
seconds (or a store that no longer answers) is reported once to ``on_failure``
from a background thread; the usual reaction is ``Model.tp_abort()``
(ncclCommAbort), after which every call on the model fails at once and
``close()`` does not wait for the lost rank. The reference has no counterpart:
its sharding (crates/wasm-chord-runtime/src/sharding.rs) is bookkeeping only.
"""
from __future__ import annotations

import threading
import time
from typing import Callable, Optional


class Watchdog:
    def __init__(self, store, rank: int, world: int, on_failure: Callable[[int], None],
                 interval: float = 0.2, timeout: float = 2.0, prefix: str = "wcb_tp_heartbeat"):
        if timeout <= interval:
            raise ValueError("timeout must exceed the heartbeat interval")
        self.store, self.rank, self.world = store, rank, world
        self.on_failure, self.interval, self.timeout, self.prefix = on_failure, interval, timeout, prefix
        self.failed_rank: Optional[int] = None
        self._stop = threading.Event()
        self._fired = threading.Event()
        self._thread = threading.Thread(target=self._run, name=f"wcb-watchdog-{rank}", daemon=True)

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def start(self) -> "Watchdog":
        self.store.add(self._key(self.rank), 1)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread.is_alive():
            self._thread.join(timeout=5 * self.interval + 1.0)

    def wait_failure(self, timeout: float) -> Optional[int]:
        """The failed rank once one was reported, or None after `timeout` seconds."""
        self._fired.wait(timeout)
        return self.failed_rank

    def _fire(self, r: int) -> None:
        self.failed_rank = r
        self._fired.set()
        try:
            self.on_failure(r)
        finally:
            self._stop.set()

    def _run(self) -> None:
        now = time.monotonic()
        seen = {r: (-1, now) for r in range(self.world) if r != self.rank}
        while not self._stop.wait(self.interval):
            try:
                self.store.add(self._key(self.rank), 1)
                now = time.monotonic()
                for r, (last, at) in list(seen.items()):
                    v = self.store.add(self._key(r), 0)  # reads without blocking
                    if v != last:
                        seen[r] = (v, now)
                    elif now - at > self.timeout:
                        self._fire(r)
                        return
            except Exception:  # the store's host (rank 0) is gone
                self._fire(0 if self.rank != 0 else -1)
                return
