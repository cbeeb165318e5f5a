"""Host-side failure detection for multi-rank serving.

Every rank runs a small monitor thread that publishes a heartbeat into a
key-value store (``torch.distributed.TCPStore``) and watches the other ranks'
heartbeats and failure markers.  A rank that raises publishes its error
(``Health.fail``) before it leaves; a rank that dies silently stops beating.
The engine calls ``Health.check()`` before it launches a step's kernels, so the
surviving ranks learn of a failure on the host between steps -- never by
spinning on a device flag -- and raise ``PeerFailure``.  A short process-group
timeout bounds any collective already waiting on the lost rank.

Device-side waits are bounded separately (every peer-flag spin in the fused
kernels gives up after a %globaltimer budget and reports kErrPeerTimeout).

There is no elastic recovery: as in the reference, a faulted rank group is torn
down and restarted (engines/glm5-moe-nvfp4-2b/src/fabric/rdma.cc:40-52 bounded
waits; engines/qwen38-flash-next-nvfp4-2b/src/decode/execution.h:29,78-82
terminal Faulted state).
"""
from __future__ import annotations

import threading
import time


class PeerFailure(RuntimeError):
    def __init__(self, failed: dict):
        self.failed = dict(failed)
        super().__init__("peer rank(s) failed: " + "; ".join(f"rank {r}: {m}" for r, m in sorted(failed.items())))


class Health:
    def __init__(self, store, rank: int, world: int, interval_s: float = 0.25, max_age_s: float = 2.0,
                 prefix: str = "rkt_health", startup_grace_s: float = 60.0):
        self.store = store
        self.rank, self.world = rank, world
        self.interval = interval_s
        self.max_age = max_age_s
        self.prefix = prefix
        self.grace = startup_grace_s  # a rank that never beat yet is still starting up
        self._failed: dict[int, str] = {}
        self._lock = threading.Lock()
        self._io = threading.Lock()  # one store request at a time (main thread and monitor)
        self._stop = threading.Event()
        self._seen: dict[int, tuple[str, float]] = {}  # last heartbeat value and when it changed (local clock)
        self._started = time.monotonic()
        self._beat = 0
        self.beat()
        self._thread = threading.Thread(target=self._run, name="rkt-health", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------------ publishing
    def beat(self):
        with self._io:
            self._beat += 1
            self.store.set(f"{self.prefix}/hb/{self.rank}", str(self._beat))

    def fail(self, msg: str):
        """Publish this rank's failure (call from an exception handler before leaving)."""
        try:
            with self._io:
                self.store.set(f"{self.prefix}/fail/{self.rank}", str(msg)[:500])
        except Exception:
            pass

    def close(self):
        self._stop.set()
        self._thread.join(timeout=5)

    # ------------------------------------------------------------------ watching
    def _poll(self):
        with self._io:
            self._poll_locked()

    def _poll_locked(self):
        now = time.monotonic()
        for r in range(self.world):
            if r == self.rank or r in self._failed:
                continue
            fk = f"{self.prefix}/fail/{r}"
            if self.store.check([fk]):
                self._mark(r, self.store.get(fk).decode(errors="replace"))
                continue
            hk = f"{self.prefix}/hb/{r}"
            val = self.store.get(hk).decode() if self.store.check([hk]) else None
            last = self._seen.get(r)
            if last is None or last[0] != val:
                self._seen[r] = (val, now)
            elif val is None:
                if now - self._started > self.grace:
                    self._mark(r, f"never started within {self.grace:.0f} s")
            elif now - last[1] > self.max_age:
                self._mark(r, f"no heartbeat for {now - last[1]:.1f} s")

    def _mark(self, r, msg):
        with self._lock:
            self._failed[r] = msg

    def _run(self):
        while not self._stop.wait(self.interval):
            try:
                self.beat()
                self._poll()
            except Exception as e:  # the store itself went away (rank 0 died): everyone is failed
                self._mark(-1, f"health store unreachable: {e}")

    def failed(self) -> dict:
        with self._lock:
            return dict(self._failed)

    def check(self):
        """Raise PeerFailure if any other rank failed (cheap: reads local state only)."""
        f = self.failed()
        if f:
            raise PeerFailure(f)


def from_env(rank: int, world: int, port_offset: int = 1, **kw) -> Health:
    """Health monitor on a TCPStore at MASTER_ADDR:MASTER_PORT+port_offset (rank 0 hosts)."""
    import datetime
    import os

    from torch.distributed import TCPStore
    host = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ.get("MASTER_PORT", "29500")) + port_offset
    store = TCPStore(host, port, world, rank == 0, timeout=datetime.timedelta(seconds=30),
                     wait_for_workers=False)
    return Health(store, rank, world, **kw)
