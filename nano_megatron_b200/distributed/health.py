"""Host-side failure detection between training ranks (no GPU involvement).

Every rank publishes a heartbeat (wall-clock seconds) under ``<prefix>/hb/<rank>`` in the
job's c10d key-value store from a daemon thread, and a rank whose step raises writes
``<prefix>/failed/<rank>`` = the error before it exits. Before launching each step a rank
calls :meth:`PeerHealth.check`, which raises :class:`PeerFailure` naming the failed or
silent ranks -- so the survivors stop on the host, between steps, instead of entering a
collective that their peer will never join. Kernels never wait on this: the device side
relies on its own bounded waits.

The reference has no heartbeat or failure marker (its README lists elastic recovery as
out of scope); it relies on the process-group timeout alone, which is kept here too.
"""

from __future__ import annotations

import threading
import time


class PeerFailure(RuntimeError):
    """Another rank failed or stopped sending heartbeats."""


class PeerHealth:
    def __init__(self, store, rank: int, world: int, *, interval_s: float = 5.0,
                 stale_s: float = 120.0, prefix: str = "nmb/health") -> None:
        if interval_s <= 0 or stale_s <= interval_s:
            raise ValueError("need 0 < interval_s < stale_s")
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.interval_s, self.stale_s, self.prefix = float(interval_s), float(stale_s), prefix
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    @classmethod
    def from_default_group(cls, **kw) -> "PeerHealth | None":
        import torch.distributed as dist

        if not (dist.is_available() and dist.is_initialized()):
            return None
        from torch.distributed import distributed_c10d as c10d

        return cls(c10d._get_default_store(), dist.get_rank(), dist.get_world_size(), **kw)

    # ------------------------------------------------------------------ publishing
    def beat(self) -> None:
        self.store.set(f"{self.prefix}/hb/{self.rank}", repr(time.time()))

    def start(self) -> "PeerHealth":
        self.beat()
        if self._thread is None:
            def loop():
                while not self._stop.wait(self.interval_s):
                    try:
                        self.beat()
                    except Exception:  # noqa: BLE001 - store gone at shutdown
                        return

            self._thread = threading.Thread(target=loop, name="nmb-heartbeat", daemon=True)
            self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=self.interval_s + 1.0)
            self._thread = None

    def report_failure(self, error: BaseException | str) -> None:
        try:
            self.store.set(f"{self.prefix}/failed/{self.rank}", str(error)[:2000] or "failed")
        except Exception:  # noqa: BLE001 - best effort while failing
            pass

    # ------------------------------------------------------------------ checking
    def _get(self, key: str) -> str | None:
        if not self.store.check([key]):
            return None
        return self.store.get(key).decode("utf-8", "replace")

    def check(self, now: float | None = None) -> None:
        """Raise PeerFailure if any other rank reported a failure or went silent."""
        now = time.time() if now is None else now
        failed, silent = [], []
        for r in range(self.world):
            if r == self.rank:
                continue
            msg = self._get(f"{self.prefix}/failed/{r}")
            if msg is not None:
                failed.append(f"rank {r}: {msg}")
                continue
            hb = self._get(f"{self.prefix}/hb/{r}")
            if hb is not None and now - float(hb) > self.stale_s:
                silent.append(f"rank {r} silent for {now - float(hb):.0f}s")
        if failed or silent:
            raise PeerFailure("; ".join(failed + silent))
