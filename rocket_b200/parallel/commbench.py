"""Communication microbenchmark at the engine's message sizes.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 -m rocket_b200.parallel.commbench

For each size: NCCL all-reduce, all-gather, reduce-scatter, all-to-all and
broadcast (torch.distributed over NCCL), and a peer-write probe -- this build's
own vector-store kernel writing into the next rank's CUDA-IPC-mapped memory (the
transport the fused collectives use).  Device time by CUDA events, max over
ranks; algorithm bandwidth = bytes / time and NCCL-convention bus bandwidth.

Counterpart of the reference's fabric microbenchmark at the decode step's
message sizes (engines/glm5-moe-nvfp4-2b/src/fabric/fabric_bench.cu).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

SIZES = [4 << 10, 64 << 10, 512 << 10, 4 << 20, 32 << 20, 256 << 20]


def _time(fn, par, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return par.max_over_ranks(a.elapsed_time(b) / iters)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes", default=",".join(str(s) for s in SIZES))
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    from .. import ops
    from .context import init_from_env
    from .symm import SymmetricHeap
    par = init_from_env(timeout_s=120)
    N, r, dev = par.world, par.rank, par.device
    if N < 2:
        raise SystemExit("commbench needs >= 2 ranks (torchrun)")
    sizes = [int(x) for x in a.sizes.split(",")]
    heap = SymmetricHeap(par, max(sizes) + (1 << 20), slot=0)
    dst_off = heap.alloc(max(sizes))
    rows = []
    for nb in sizes:
        n = nb // 2  # bf16 elements
        x = torch.randn(n, device=dev).bfloat16()
        y = torch.empty(n * N, device=dev, dtype=torch.bfloat16)
        z = torch.empty(max(n // N, 1), device=dev, dtype=torch.bfloat16)
        res = {"bytes": nb}
        t = _time(lambda: dist.all_reduce(x), par, a.iters)
        res["all_reduce_ms"], res["all_reduce_busbw_gbs"] = round(t, 4), round(nb / t / 1e6 * 2 * (N - 1) / N, 1)
        t = _time(lambda: dist.all_gather_into_tensor(y, x), par, a.iters)
        res["all_gather_ms"], res["all_gather_busbw_gbs"] = round(t, 4), round(nb * N / t / 1e6 * (N - 1) / N, 1)
        if n % N == 0:
            t = _time(lambda: dist.reduce_scatter_tensor(z, x), par, a.iters)
            res["reduce_scatter_ms"], res["reduce_scatter_busbw_gbs"] = round(t, 4), round(nb / t / 1e6 * (N - 1) / N, 1)
            xa = torch.empty_like(x)
            t = _time(lambda: dist.all_to_all_single(xa, x), par, a.iters)
            res["all_to_all_ms"], res["all_to_all_busbw_gbs"] = round(t, 4), round(nb / t / 1e6 * (N - 1) / N, 1)
        t = _time(lambda: dist.broadcast(x, 0), par, a.iters)
        res["broadcast_ms"] = round(t, 4)
        peer = heap.bases[(r + 1) % N] + dst_off
        t = _time(lambda: ops.ext().p2p_copy(x, peer, nb, 296), par, a.iters)
        res["peer_write_ms"], res["peer_write_gbs"] = round(t, 4), round(nb / t / 1e6, 1)
        rows.append(res)
    if r == 0:
        print(json.dumps({"bench": "commbench", "n_gpus": N, "timing": "CUDA events, max over ranks",
                          "results": rows}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
