"""Multi-rank state transactions on gloo CPU ranks: commit, authenticated restore, and
crashes injected at every protocol phase (host-side failures only)."""
import datetime
import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

WORLD = 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _parts(rank, gen):
    rng = np.random.default_rng(100 * gen + rank)
    return [rng.integers(0, 255, 1000 + 37 * rank, dtype=np.uint8),
            rng.standard_normal(64).astype(np.float32)]


def _worker(rank, port, root, crash_phase, crash_rank, q):
    import torch.distributed as dist

    from rocket_b200.kv.state_txn import DistributedTxn, TxnError
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=30))
    try:
        armed = {"on": False}

        def fault(phase):
            if armed["on"] and rank == crash_rank and phase == crash_phase:
                raise RuntimeError(f"injected crash at {phase}")

        tx = DistributedTxn(root, fault=fault)
        tx.checkpoint("s1", _parts(rank, 1))            # generation 1 commits everywhere
        armed["on"] = True
        outcome = "committed"
        try:
            tx.checkpoint("s1", _parts(rank, 2))        # generation 2 meets the crash
        except TxnError:
            outcome = "aborted"
        except RuntimeError:
            outcome = "crashed"
        armed["on"] = False
        # the crashed rank "restarts": a fresh store on the same directory
        tx = DistributedTxn(root)
        txn, parts = tx.restore("s1")
        gen = None
        for g in (1, 2):
            exp = _parts(rank, g)
            if all(np.array_equal(a.view(np.uint8), np.ascontiguousarray(b).view(np.uint8).reshape(-1))
                   for a, b in zip(parts, exp)):
                gen = g
        q.put((rank, outcome, gen))
    finally:
        dist.destroy_process_group()


# phase -> generation every rank must restore after a crash of rank 1 there
EXPECT = {None: 2, "prepare": 1, "vote": 1, "commit": 1, "index": 2, "cleanup": 2}


@pytest.mark.parametrize("phase", list(EXPECT))
def test_crash_at_every_phase_restores_a_consistent_generation(tmp_path, phase):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, str(tmp_path), phase, 1, q)) for r in range(WORLD)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(WORLD))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    gens = {g for _, _, g in res}
    assert gens == {EXPECT[phase]}, res   # every rank on the same, complete generation


def test_tampered_decision_and_payload_are_refused(tmp_path):
    from rocket_b200.kv.state_txn import DistributedTxn, TxnError
    tx = DistributedTxn(str(tmp_path))           # world 1 (no process group)
    t1 = tx.checkpoint("a", _parts(0, 1))
    t2 = tx.checkpoint("a", _parts(0, 2))
    assert tx.restore("a")[0] == t2
    # a forged decision record (tag no longer matches) -> the previous transaction
    cp = os.path.join(str(tmp_path), "rank0", f"txn-{t2}", "COMMIT")
    rec = json.load(open(cp))
    rec["receipts"][0]["sizes"][0] += 0
    rec["session"] = "a"
    rec["time_ns"] += 1
    open(cp, "w").write(json.dumps(rec))
    assert tx.restore("a")[0] == t1
    # damaged payload of the remaining one -> nothing restorable
    pp = os.path.join(str(tmp_path), "rank0", f"txn-{t1}", "payload")
    b = bytearray(open(pp, "rb").read())
    b[5] ^= 1
    open(pp, "wb").write(bytes(b))
    with pytest.raises(TxnError):
        tx.restore("a")
    # a wrong deployment key cannot authenticate anything
    t3 = tx.checkpoint("b", _parts(0, 3))
    other = DistributedTxn(str(tmp_path), key=b"another-key")
    with pytest.raises(TxnError):
        other.restore("b")
    assert tx.restore("b")[0] == t3


def test_history_is_bounded_and_orphans_collected(tmp_path):
    from rocket_b200.kv.state_txn import DistributedTxn
    tx = DistributedTxn(str(tmp_path))
    for g in range(5):
        tx.checkpoint("s", _parts(0, g))
    d = os.path.join(str(tmp_path), "rank0")
    assert len([x for x in os.listdir(d) if x.startswith("txn-")]) == 2
    os.makedirs(os.path.join(d, "txn-deadbeef-00000000"))       # an unfinished prepare
    DistributedTxn(str(tmp_path))
    assert not os.path.exists(os.path.join(d, "txn-deadbeef-00000000"))
