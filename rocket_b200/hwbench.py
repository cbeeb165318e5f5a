"""Device facts and memory microbenchmarks (copy / read / triad / 64-byte gather, capacity).

    python -m rocket_b200.hwbench [--sizes-mib 64,1024,4096] [--iters 20]

Each kernel is timed with CUDA events on the launching stream after warm-up,
with an L2-sized scrub between iterations for sizes below 4x L2; bandwidth counts
the algorithmic bytes (copy: read + write; read: read; triad: 2 reads + write;
gather: indices + rows read + write).  Capacity reports free / total memory and
the largest single allocation that succeeded (binary search, bounded by free).

Counterpart of the reference's hardware probes (scripts/hardware/mem-bw.cu,
mem-bw-sweep.cu, mem-gather.cu, gpu-capacity.cu) on sm_100a kernels of this
package (csrc/probe.cu).
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops

KINDS = {"copy": 0, "read": 1, "triad": 2, "gather": 3}


def _time(fn, iters: int, scrub: torch.Tensor | None) -> float:
    for _ in range(3):
        fn()
    total = 0.0
    for _ in range(iters):
        if scrub is not None:
            scrub.add_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        total += a.elapsed_time(b)
    return total / iters


def bandwidth(kind: str, nbytes: int, iters: int = 20, dev="cuda") -> dict:
    """GB/s of one kernel over `nbytes` per stream."""
    ext = ops.ext()
    nbytes = nbytes // 64 * 64
    u8 = dict(dtype=torch.uint8, device=dev)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    scrub = torch.empty(2 * l2 // 4, dtype=torch.float32, device=dev) if nbytes < 4 * l2 else None
    k = KINDS[kind]
    if kind == "gather":
        src = torch.randint(0, 255, (nbytes,), **u8)
        rows = nbytes // 64
        idx = torch.randint(0, rows, (rows,), dtype=torch.int32, device=dev)
        out = torch.empty(nbytes, **u8)
        fn = lambda: ext.mem_bw(k, out, src, None, idx, nbytes)
        moved = nbytes * 2 + rows * 4
    else:
        b = torch.randint(0, 255, (nbytes,), **u8)
        c = torch.randint(0, 255, (nbytes,), **u8) if kind == "triad" else None
        a = torch.empty(nbytes if kind != "read" else 64, **u8)
        fn = lambda: ext.mem_bw(k, a, b, c, None, nbytes)
        moved = {"copy": 2, "read": 1, "triad": 3}[kind] * nbytes
    ms = _time(fn, iters, scrub)
    return {"kernel": kind, "bytes": nbytes, "ms": round(ms, 4), "gb_s": round(moved / ms / 1e6, 1)}


def capacity(dev="cuda") -> dict:
    free, total = torch.cuda.mem_get_info(dev)
    lo, hi = 0, free
    step = 1 << 30
    while hi - lo > step:
        mid = (lo + hi) // 2 // step * step
        try:
            t = torch.empty(mid, dtype=torch.uint8, device=dev)
            del t
            torch.cuda.empty_cache()
            lo = mid
        except torch.OutOfMemoryError:
            hi = mid
    return {"free_gib": round(free / 2**30, 2), "total_gib": round(total / 2**30, 2),
            "largest_alloc_gib": round(lo / 2**30, 2)}


def facts(dev="cuda") -> dict:
    p = torch.cuda.get_device_properties(dev)
    return {"name": p.name, "sm": f"{p.major}.{p.minor}", "sms": p.multi_processor_count,
            "l2_mib": p.L2_cache_size >> 20, "total_gib": round(p.total_memory / 2**30, 1)}


def main(argv=None):
    ap = argparse.ArgumentParser(prog="rocket_b200.hwbench")
    ap.add_argument("--sizes-mib", default="64,1024,4096")
    ap.add_argument("--kinds", default="copy,read,triad,gather")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--capacity", action="store_true", help="also probe the largest allocation")
    a = ap.parse_args(argv)
    out = {"device": facts(), "bandwidth": []}
    for mib in [int(x) for x in a.sizes_mib.split(",")]:
        for kind in a.kinds.split(","):
            out["bandwidth"].append(bandwidth(kind, mib << 20, a.iters))
            torch.cuda.empty_cache()
    if a.capacity:
        out["capacity"] = capacity()
    print(json.dumps(out))


if __name__ == "__main__":
    main()
