"""Peer heartbeat watchdog (host side).

Each rank runs a daemon thread that stamps ``hb/<rank>`` in a shared
``torch.distributed`` store every ``period_s`` and reads every peer's stamp.
A peer whose stamp is older than ``timeout_s`` (or missing after the grace
period) is reported dead: ``dead_peers()`` lists it and ``on_dead`` is called
once per peer.  Runtimes check it between steps and stop before launching work
that would wait on the dead peer (the device waits are bounded as well).
"""

from __future__ import annotations

import threading
import time
from collections.abc import Callable

_DONE = "done"


class HeartbeatWatchdog:
    def __init__(self, store, rank: int, world_size: int, *, period_s: float = 0.2, timeout_s: float = 2.0,
                 on_dead: Callable[[int], None] | None = None, prefix: str = "hb"):
        self.store = store
        self.rank = rank
        self.world = world_size
        self.period = period_s
        self.timeout = timeout_s
        self.on_dead = on_dead
        self.prefix = prefix
        self._dead: set[int] = set()
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._start = time.time()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self.store.set(self._key(self.rank), repr(time.time()))

    def _check(self) -> None:
        now = time.time()
        for r in range(self.world):
            if r == self.rank or r in self._dead:
                continue
            try:
                raw = self.store.get(self._key(r)).decode() if self._has(r) else None
            except Exception:  # noqa: BLE001 - store unreachable counts as stale
                raw = None
            if raw == _DONE:
                continue  # the peer left cleanly
            stamp = float(raw) if raw is not None else None
            stale = (stamp is None and now - self._start > self.timeout) or (
                stamp is not None and now - stamp > self.timeout)
            if stale:
                self._dead.add(r)
                if self.on_dead is not None:
                    self.on_dead(r)

    def _has(self, r: int) -> bool:
        try:
            return self.store.check([self._key(r)])
        except Exception:  # noqa: BLE001
            return False

    def _loop(self) -> None:
        while not self._stop.is_set():
            try:
                self.beat()
            except Exception:  # noqa: BLE001 - our own store write failing: keep checking peers
                pass
            self._check()
            self._stop.wait(self.period)

    def start(self) -> "HeartbeatWatchdog":
        self.beat()
        self._thread = threading.Thread(target=self._loop, name="afd-heartbeat", daemon=True)
        self._thread.start()
        return self

    def stop(self, *, clean: bool = True) -> None:
        """Stop beating; with ``clean`` the peers learn this rank left on purpose (no death report)."""
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.period + 1)
        if clean:
            try:
                self.store.set(self._key(self.rank), _DONE)
            except Exception:  # noqa: BLE001 - the store may already be gone at exit
                pass

    def dead_peers(self) -> set[int]:
        return set(self._dead)

    def raise_if_peer_dead(self) -> None:
        if self._dead:
            raise RuntimeError(f"AFD peer rank(s) {sorted(self._dead)} stopped heartbeating")


__all__ = ["HeartbeatWatchdog"]
