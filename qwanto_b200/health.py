"""Rank liveness for the multi-GPU paths (failure detection on the host).

Each rank runs a :class:`Heartbeat`: a background thread that bumps a counter
under ``<prefix>/<rank>`` in the process group's key-value store every
``interval`` seconds.  Before a step whose launches or collectives need every
rank, a rank calls :meth:`Heartbeat.check_peers`: it returns once every other
rank's counter has moved, and raises :class:`RankLostError` naming the ranks
whose counters stood still for ``timeout`` seconds.  A rank that exits or
hangs between steps -- silently, without announcing anything -- is therefore
found on the host before the next launch, instead of leaving the others
waiting inside a collective or a peer-flag wait on the GPU.

The store is the one ``torch.distributed`` already holds (TCPStore hosted by
rank 0), so this adds no connection.  If rank 0 itself is gone, the store
calls fail and :meth:`check_peers` raises as well.
"""
from __future__ import annotations

import threading
import time


class RankLostError(RuntimeError):
    """Raised when peers stopped heartbeating; ``ranks`` lists them."""

    def __init__(self, ranks, detail: str = ""):
        self.ranks = sorted(ranks)
        super().__init__(f"ranks {self.ranks} stopped heartbeating{': ' + detail if detail else ''}")


class Heartbeat:
    def __init__(self, store, rank: int, world: int, interval: float = 0.05, prefix: str = "qwn_hb"):
        if world < 1 or not 0 <= rank < world:
            raise ValueError("rank out of range")
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.prefix = float(interval), prefix
        self._beat = 0
        self._stop = threading.Event()
        self._thread = None
        self.error = None  # the exception that ended the beating thread, if any

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _run(self):
        try:
            while not self._stop.is_set():
                self._beat += 1
                self.store.set(self._key(self.rank), str(self._beat))
                self._stop.wait(self.interval)
        except Exception as e:  # the store went away (rank 0 died): report it at the next check
            self.error = e

    def start(self) -> "Heartbeat":
        self.store.set(self._key(self.rank), "0")
        self._thread = threading.Thread(target=self._run, name=f"qwn-heartbeat-{self.rank}", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval + 1.0)
            self._thread = None

    def _read(self, r: int):
        key = self._key(r)
        if not self.store.check([key]):
            return None
        return int(self.store.get(key))

    def check_peers(self, timeout: float = 2.0) -> None:
        """Return when every other rank has beaten since this call began;
        raise RankLostError for the ranks that did not within `timeout`."""
        if self.error is not None:
            raise RankLostError([0], f"store unreachable ({self.error})")
        peers = [r for r in range(self.world) if r != self.rank]
        try:
            first = {r: self._read(r) for r in peers}
            waiting = set(peers)
            deadline = time.monotonic() + timeout
            while waiting:
                for r in list(waiting):
                    v = self._read(r)
                    if v is not None and (first[r] is None or v > first[r]):
                        waiting.discard(r)
                if not waiting:
                    return
                if time.monotonic() >= deadline:
                    raise RankLostError(waiting, f"no heartbeat for {timeout:g} s")
                time.sleep(min(self.interval, 0.02))
        except RankLostError:
            raise
        except Exception as e:
            raise RankLostError([0], f"store unreachable ({e})") from e

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()
        return False
