"""Failure detection without any GPU fault: failures are made on the host among CPU
ranks (a rank that exits silently, a rank that raises, a rank that never joins a
collective) and the survivors must learn of them in bounded time.

Counterparts of the reference's fault injection (a stalled peer,
engines/qwen38-flash-next-nvfp4-2b/bench/pair_reduce_bench.cu:195-215; bounded
doorbell waits, engines/glm5-moe-nvfp4-2b/src/fabric/rdma.cc:40-52).
"""
import datetime
import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _store(rank, port):
    from torch.distributed import TCPStore
    return TCPStore("127.0.0.1", port, 2, rank == 0, timeout=datetime.timedelta(seconds=20), wait_for_workers=False)


def _health_worker(rank, port, mode, q):
    from rocket_b200.parallel.health import Health, PeerFailure
    st = _store(rank, port)
    h = Health(st, rank, 2, interval_s=0.05, max_age_s=0.6)
    if rank == 1:
        time.sleep(0.4)
        if mode == "exit":
            os._exit(0)  # dies without a word: heartbeats stop
        try:
            raise ValueError("injected step failure")
        except ValueError as e:
            h.fail(f"{type(e).__name__}: {e}")
            time.sleep(0.5)
            os._exit(1)
    t0 = time.monotonic()
    while time.monotonic() - t0 < 10:
        try:
            h.check()
        except PeerFailure as e:
            q.put(("detected", round(time.monotonic() - t0, 2), e.failed))
            h.close()
            return
        time.sleep(0.05)
    q.put(("missed", None, {}))


@pytest.mark.parametrize("mode", ["exit", "raise"])
def test_peer_failure_detected_on_host(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_health_worker, args=(r, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    what, dt, failed = q.get(timeout=60)
    for p in ps:
        p.join(timeout=30)
    assert what == "detected", what
    assert 1 in failed
    if mode == "raise":
        assert "injected step failure" in failed[1]
    assert dt < 5.0


def _pg_worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=2))
    if rank == 1:
        time.sleep(6)  # alive, but never joins the collective
        q.put((1, "slept", 0.0))
        return
    t = torch.ones(4)
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
        q.put((0, "completed", time.monotonic() - t0))
    except Exception as e:
        q.put((0, type(e).__name__, time.monotonic() - t0))


def test_collective_with_missing_rank_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_pg_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2):
        r, what, dt = q.get(timeout=60)
        res[r] = (what, dt)
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[0][0] != "completed", res
    assert res[0][1] < 5.0, res
