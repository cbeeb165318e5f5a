"""Atomic multi-rank state transactions (checkpoint / restore of sessions).

Every rank owns a local directory and writes only its own shard of a session's
state (its KV head shard, its DeltaNet heads, ...).  A checkpoint is a
collective two-phase commit:

1. prepare -- each rank writes its parts to ``txn-<id>/payload`` (fsync) and
   computes a receipt: rank, part sizes, a 256-bit digest of the bytes;
2. vote    -- the receipts are all-gathered; the transaction commits only if
   every rank prepared;
3. commit  -- each rank writes the same decision record (every receipt, the
   transaction id, an HMAC-SHA256 tag over it under a deployment key) to
   ``txn-<id>/COMMIT`` and fsyncs it;
4. index   -- each rank atomically repoints ``index/<session>`` at the
   transaction (write + rename), then deletes the transaction it replaced.

A crash anywhere leaves every rank either on the previous committed
transaction or on the new one; restore detects a mixed state (ranks whose
indexes name different transactions after a crash between step 4's renames),
and then falls back to the newest transaction that every rank still has
committed.  Restore is collective too: each rank authenticates the decision
record (HMAC), checks its payload against its own receipt, and the ranks agree
on the outcome before any of them uses the bytes.  Unreferenced or uncommitted
transaction directories are removed when a store opens.

Fault injection for tests: ``fault(phase)`` is called at every protocol step
and may raise (a crashed rank) -- the host-side failure model; nothing here
touches a GPU.

Counterpart of the reference's two-rank state transactions
(engines/qwen38-flash-next-nvfp4-2b/src/qwen38_slab/state_txn.py:229,
distributed_state_txn.py:232 -- prepare / commit / index / authenticate /
publish; crash-point tests qw/tests/test_distributed_state_txn.py:109); here for
N ranks over torch.distributed with the native digest.
"""
from __future__ import annotations

import hashlib
import hmac
import json
import os
import shutil
import time
import uuid

import numpy as np

PHASES = ("prepare", "vote", "commit", "index", "cleanup")


class TxnError(RuntimeError):
    pass


def _fsync_dir(d: str):
    fd = os.open(d, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def _atomic_write(path: str, data: bytes):
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)
    _fsync_dir(os.path.dirname(path))


def _digest(parts) -> str:
    from .. import _rt
    h = hashlib.blake2b(digest_size=32)
    for p in parts:
        b = np.ascontiguousarray(p).view(np.uint8).reshape(-1)
        h.update(len(b).to_bytes(8, "little"))
        h.update(bytes.fromhex(_rt.digest_hex(b)))
    return h.hexdigest()


def _safe(name: str) -> str:
    if not name or any(c in name for c in "/\\\0") or name.startswith("."):
        raise ValueError(f"bad session id {name!r}")
    return name


class RankTxnStore:
    """One rank's side of the protocol (local files only)."""

    def __init__(self, root: str, rank: int, key: bytes = b"rocket_b200-default-key", fault=None):
        self.rank = rank
        self.dir = os.path.join(root, f"rank{rank}")
        self.key = key
        self.fault = fault or (lambda phase: None)
        os.makedirs(os.path.join(self.dir, "index"), exist_ok=True)
        self._gc()

    # ---------------------------------------------------------------- files
    def _tdir(self, txn: str) -> str:
        return os.path.join(self.dir, f"txn-{txn}")

    def _index(self, session: str) -> str:
        return os.path.join(self.dir, "index", _safe(session))

    def _tag(self, decision: dict) -> str:
        body = json.dumps(decision, sort_keys=True, separators=(",", ":")).encode()
        return hmac.new(self.key, body, hashlib.sha256).hexdigest()

    def _gc(self):
        """Drop transactions no index names, unless they are committed and newer than
        every index entry (kept as restore fallbacks: a crash between the ranks'
        index renames leaves one of them pointing at the other's old txn)."""
        live = set()
        idx = os.path.join(self.dir, "index")
        for s in os.listdir(idx):
            if s.endswith(".tmp"):
                os.unlink(os.path.join(idx, s))
                continue
            with open(os.path.join(idx, s)) as f:
                live.update(json.load(f)["history"])
        for d in os.listdir(self.dir):
            if d.startswith("txn-") and d[4:] not in live:
                if not os.path.exists(os.path.join(self.dir, d, "COMMIT")):
                    shutil.rmtree(os.path.join(self.dir, d), ignore_errors=True)

    # ---------------------------------------------------------------- protocol
    def prepare(self, session: str, txn: str, parts: list[np.ndarray]) -> dict:
        self.fault("prepare")
        d = self._tdir(txn)
        os.makedirs(d)
        sizes = [int(np.asarray(p).nbytes) for p in parts]
        with open(os.path.join(d, "payload"), "wb") as f:
            for p in parts:
                f.write(np.ascontiguousarray(p).view(np.uint8).reshape(-1).tobytes())
            f.flush()
            os.fsync(f.fileno())
        _fsync_dir(d)
        return {"rank": self.rank, "session": session, "txn": txn, "sizes": sizes, "digest": _digest(parts)}

    def commit(self, decision: dict):
        self.fault("commit")
        rec = dict(decision, tag=self._tag(decision))
        _atomic_write(os.path.join(self._tdir(decision["txn"]), "COMMIT"),
                      json.dumps(rec, sort_keys=True).encode())

    def index(self, session: str, txn: str, keep: int = 2):
        self.fault("index")
        p = self._index(session)
        hist = []
        if os.path.exists(p):
            with open(p) as f:
                hist = json.load(f)["history"]
        hist = [txn] + [h for h in hist if h != txn]
        _atomic_write(p, json.dumps({"session": session, "history": hist[:keep]}).encode())
        self.fault("cleanup")
        for old in hist[keep:]:
            shutil.rmtree(self._tdir(old), ignore_errors=True)

    def abort(self, txn: str):
        shutil.rmtree(self._tdir(txn), ignore_errors=True)

    def history(self, session: str) -> list[str]:
        p = self._index(session)
        if not os.path.exists(p):
            return []
        with open(p) as f:
            return json.load(f)["history"]

    def committed(self, session: str) -> list[str]:
        """Committed transactions of `session` on this rank, newest first (the index
        history, then committed orphans newer than it)."""
        out = []
        for d in os.listdir(self.dir):
            cp = os.path.join(self.dir, d, "COMMIT")
            if d.startswith("txn-") and os.path.exists(cp):
                with open(cp) as f:
                    rec = json.load(f)
                if rec.get("session") == session:
                    out.append((rec["time_ns"], d[4:]))
        return [t for _, t in sorted(out, reverse=True)]

    def authenticate(self, session: str, txn: str, world: int) -> tuple[bool, str]:
        """(ok, decision digest) for this rank's view of transaction `txn`."""
        try:
            with open(os.path.join(self._tdir(txn), "COMMIT")) as f:
                rec = json.load(f)
            tag = rec.pop("tag")
            if not hmac.compare_digest(tag, self._tag(rec)):
                return False, "bad-tag"
            if rec["session"] != session or rec["txn"] != txn or len(rec["receipts"]) != world:
                return False, "mismatch"
            mine = rec["receipts"][self.rank]
            parts = self._read_parts(txn, mine["sizes"])
            if _digest(parts) != mine["digest"]:
                return False, "bad-payload"
            return True, hashlib.sha256(json.dumps(rec, sort_keys=True).encode()).hexdigest()
        except (OSError, ValueError, KeyError, IndexError):
            return False, "missing"

    def _read_parts(self, txn: str, sizes: list[int]) -> list[np.ndarray]:
        with open(os.path.join(self._tdir(txn), "payload"), "rb") as f:
            raw = np.frombuffer(f.read(), dtype=np.uint8)
        if raw.nbytes != sum(sizes):
            raise ValueError("payload size")
        out, o = [], 0
        for s in sizes:
            out.append(raw[o:o + s].copy())
            o += s
        return out

    def read(self, txn: str) -> list[np.ndarray]:
        with open(os.path.join(self._tdir(txn), "COMMIT")) as f:
            rec = json.load(f)
        return self._read_parts(txn, rec["receipts"][self.rank]["sizes"])


class DistributedTxn:
    """Collective checkpoint / restore over a process group (every rank calls)."""

    def __init__(self, root: str, group=None, key: bytes | None = None, fault=None):
        import torch.distributed as dist
        self.dist = dist if dist.is_available() and dist.is_initialized() else None
        self.group = group
        self.rank = self.dist.get_rank(group) if self.dist else 0
        self.world = self.dist.get_world_size(group) if self.dist else 1
        key = key if key is not None else os.environ.get("ROCKET_STATE_KEY", "rocket_b200-default-key").encode()
        self.store = RankTxnStore(root, self.rank, key, fault)

    def _gather(self, obj):
        if self.dist is None:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj, group=self.group)
        return out

    def _bcast(self, obj):
        if self.dist is None:
            return obj
        box = [obj]
        self.dist.broadcast_object_list(box, src=0, group=self.group)
        return box[0]

    def checkpoint(self, session: str, parts: list[np.ndarray]) -> str:
        """Commit `parts` (this rank's shard) as the new state of `session` on every rank,
        or leave every rank on its previous state.  Returns the transaction id."""
        txn = self._bcast(f"{time.time_ns():x}-{uuid.uuid4().hex[:8]}")
        receipt, err = None, None
        try:
            receipt = self.store.prepare(session, txn, parts)
        except Exception as e:  # this rank failed to prepare: vote no
            err = f"{type(e).__name__}: {e}"
        votes = self._gather({"rank": self.rank, "receipt": receipt, "error": err})
        self.store.fault("vote")
        failed = [v for v in votes if v["receipt"] is None]
        if failed:
            self.store.abort(txn)
            raise TxnError(f"checkpoint {session}: ranks {[v['rank'] for v in failed]} failed to prepare: "
                           f"{failed[0]['error']}")
        decision = {"session": session, "txn": txn, "time_ns": int(txn.split("-")[0], 16),
                    "receipts": [v["receipt"] for v in sorted(votes, key=lambda v: v["rank"])]}
        self.store.commit(decision)
        self.store.index(session, txn)
        return txn

    def restore(self, session: str) -> tuple[str, list[np.ndarray]]:
        """This rank's parts of the newest transaction of `session` that every rank has
        committed and authenticated.  Raises if there is none."""
        mine = self.store.committed(session)
        views = self._gather(mine)
        common = [t for t in views[0] if all(t in v for v in views[1:])]
        for txn in common:  # newest first
            ok, dg = self.store.authenticate(session, txn, self.world)
            res = self._gather((ok, dg))
            if all(r[0] for r in res) and len({r[1] for r in res}) == 1:
                return txn, self.store.read(txn)
        raise TxnError(f"no committed state of {session} that every rank can authenticate")
