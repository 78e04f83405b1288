"""Independent separation windows across GPUs: one process per GPU, no
collectives on the data path.

Windows (120 s mixtures cut by the caller, triton/README.md:134-135) are
independent, so rank r of N takes windows r, r+N, r+2N, ... and runs the
attention hot path on its own device. Coordination goes through a
``torch.distributed`` key-value store (TCPStore): each rank publishes one small
record per finished window and a heartbeat; rank 0 collects the records. A rank
that raises, exits or stops beating is detected on the host (its windows are
missing after the deadline and its heartbeat is stale) and its unfinished
windows are re-run by the surviving ranks. No kernel or collective is in
flight when a rank leaves: failure handling is host-only.
"""

from __future__ import annotations

import json
import threading
import time
from dataclasses import dataclass, field
from typing import Callable


def assign(n_windows: int, world: int) -> list[list[int]]:
    """Round-robin partition of window ids over ranks."""
    return [list(range(r, n_windows, world)) for r in range(world)]


@dataclass
class RunReport:
    results: dict[int, object] = field(default_factory=dict)   # window -> record (rank 0)
    failed_ranks: list[int] = field(default_factory=list)      # ranks detected as gone
    requeued: dict[int, int] = field(default_factory=dict)     # window -> rank that re-ran it
    wall_s: float = 0.0


class WindowRunner:
    """Runs ``process(window_id) -> JSON-serialisable record`` over all windows.

    store:      a torch.distributed Store shared by every rank
    heartbeat_s: how often a rank refreshes its heartbeat key
    dead_after_s: a rank whose heartbeat is older than this, with windows
                 still missing, is declared failed
    window_timeout_s: a background thread keeps the heartbeat fresh while
                 ``process`` runs, for at most this long per window; a window
                 that takes longer stops the heartbeat (treated as hung)
    start_grace_s: a rank that has not published its first heartbeat yet is
                 "not started", not failed, until this long after the
                 observer started (slow process start-up, lazy CUDA init)
    deadline_s:  overall bound for the whole run (raises TimeoutError)
    """

    def __init__(self, store, rank: int, world: int, n_windows: int, *, prefix: str = "fds/win",
                 heartbeat_s: float = 0.2, dead_after_s: float = 3.0, window_timeout_s: float = 300.0,
                 start_grace_s: float = 60.0, deadline_s: float = 600.0):
        self.store, self.rank, self.world, self.n = store, rank, world, n_windows
        self.prefix = prefix
        self.heartbeat_s, self.dead_after_s, self.deadline_s = heartbeat_s, dead_after_s, deadline_s
        self.window_timeout_s, self.start_grace_s = window_timeout_s, start_grace_s
        self._last_beat = 0.0
        self._t0 = time.time()
        self._lock = threading.Lock()   # the store client is shared with the heartbeat thread

    # ---------------------------------------------------------------- keys
    def _k(self, *parts) -> str:
        return "/".join([self.prefix, *map(str, parts)])

    def _set(self, key: str, value: str) -> None:
        with self._lock:
            self.store.set(key, value)

    def _get(self, key: str) -> bytes:
        with self._lock:
            return self.store.get(key)

    def _has(self, key: str) -> bool:
        with self._lock:
            return self.store.check([key])

    def _add(self, key: str, n: int) -> int:
        with self._lock:
            return self.store.add(key, n)

    def _beat(self, force: bool = False) -> None:
        now = time.time()
        if force or now - self._last_beat >= self.heartbeat_s:
            self._set(self._k("hb", self.rank), repr(now))
            self._last_beat = now

    def _done(self, w: int) -> bool:
        return self._has(self._k("done", w))

    def _publish(self, w: int, record) -> None:
        self._set(self._k("done", w), json.dumps({"rank": self.rank, "record": record}))

    def _alive(self, r: int) -> bool:
        key = self._k("hb", r)
        if self._has(self._k("fin", r)):
            return True
        if not self._has(key):
            # not started yet: failed only once the start grace period is over
            return time.time() - self._t0 < self.start_grace_s
        return time.time() - float(self._get(key).decode()) < self.dead_after_s

    def _process(self, process: Callable[[int], object], w: int):
        """Runs process(w) while a background thread keeps the heartbeat fresh
        (for at most window_timeout_s: a hung window then goes quiet)."""
        stop = threading.Event()
        started = time.time()

        def keep_beating():
            while not stop.wait(self.heartbeat_s):
                if time.time() - started > self.window_timeout_s:
                    return
                self._beat(force=True)

        t = threading.Thread(target=keep_beating, daemon=True)
        t.start()
        try:
            return process(w)
        finally:
            stop.set()
            t.join()

    # ---------------------------------------------------------------- run
    def run(self, process: Callable[[int], object]) -> RunReport:
        t0 = time.time()
        self._t0 = t0
        report = RunReport()
        self._beat(force=True)
        for w in assign(self.n, self.world)[self.rank]:
            self._publish(w, self._process(process, w))
            self._beat()
        self._set(self._k("fin", self.rank), "1")
        self._beat(force=True)

        # every rank then helps with windows of ranks that failed: a window is
        # claimed with an atomic counter so exactly one survivor re-runs it
        while True:
            if time.time() - t0 > self.deadline_s:
                raise TimeoutError(f"rank {self.rank}: windows still missing after {self.deadline_s} s")
            missing = [w for w in range(self.n) if not self._done(w)]
            if not missing:
                break
            progressed = False
            for w in missing:
                owner = w % self.world
                if owner == self.rank or self._alive(owner):
                    continue
                if self._add(self._k("claim", w), 1) == 1:
                    self._publish(w, self._process(process, w))
                    self._set(self._k("requeued", w), str(self.rank))
                    progressed = True
                self._beat()
            if not progressed:
                time.sleep(self.heartbeat_s / 2)
                self._beat()

        if self.rank == 0:
            for w in range(self.n):
                rec = json.loads(self._get(self._k("done", w)).decode())
                report.results[w] = rec["record"]
                if self._has(self._k("requeued", w)):
                    report.requeued[w] = int(self._get(self._k("requeued", w)).decode())
            report.failed_ranks = sorted({w % self.world for w in report.requeued})
        report.wall_s = time.time() - t0
        return report
