"""Host-side collective plumbing on CPU ranks (gloo, world_size 2): the signed
MAX trick of the vocab-parallel argmax keys, rank-0-authoritative decisions and
the shard arithmetic."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _orderable(x: float) -> int:
    import struct
    b = struct.unpack("<I", struct.pack("<f", x))[0]
    return (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from rocket_b200.parallel.context import ParallelCtx
    dist.init_process_group("gloo", rank=rank, world_size=world)
    par = ParallelCtx(rank, world, torch.device("cpu"))
    # each rank's best (value, global id) for 3 tokens; ties resolve to the lower id
    vals = {0: [(1.5, 3), (-2.0, 7), (0.25, 10)], 1: [(0.5, 103), (-1.0, 107), (0.25, 5)]}[rank]
    u64 = [(_orderable(v) << 32) | ((~i) & 0xFFFFFFFF) for v, i in vals]
    keys = torch.tensor([k - (1 << 64) if k >= (1 << 63) else k for k in u64], dtype=torch.int64)
    keys.bitwise_xor_(-(1 << 63))
    par.all_reduce_max(keys)
    keys.bitwise_xor_(-(1 << 63))
    ids = [(~int(k)) & 0xFFFFFFFF for k in keys.tolist()]
    dec = torch.tensor([rank * 10 + 1, rank * 10 + 2])
    par.broadcast(dec, 0)
    lo, hi = par.shard(160, "experts")
    q.put((rank, ids, dec.tolist(), (lo, hi)))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r, i, d, s = q.get(timeout=60)
        res[r] = (i, d, s)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        ids, dec, _ = res[r]
        assert ids == [3, 107, 5]   # max value; on an exact tie the lower id
        assert dec == [1, 2]        # rank 0 decides
    assert res[0][2] == (0, 80) and res[1][2] == (80, 160)


def test_layouts():
    """tp / ep layouts over one world: replicated dimensions keep the full extent on every
    rank; tp = ep = 1 on several ranks means the default tp = ep = world."""
    import pytest

    from rocket_b200.parallel.context import ParallelCtx
    par = ParallelCtx(1, 4, torch.device("cpu"))
    exact = par.with_layout(1, 4)
    assert (exact.tp, exact.tp_rank, exact.ep, exact.ep_rank) == (1, 0, 4, 1)
    assert exact.shard(128, "heads") == (0, 128)  # attention replicated
    full = par.with_layout(4, 4)
    assert (full.tp, full.tp_rank, full.ep, full.ep_rank) == (4, 1, 4, 1)
    assert full.shard(128, "heads") == (32, 64)
    dflt = par.with_layout(1, 1)
    assert (dflt.tp, dflt.ep) == (4, 4)
    with pytest.raises(ValueError):
        par.with_layout(2, 4)
