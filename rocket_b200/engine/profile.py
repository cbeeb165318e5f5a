"""Per-stage GPU time of one decode step (CUDA-event stage timer, eager launch).

``profile_decode(engine, batch, ctx)`` opens `batch` synthetic sequences whose
KV holds `ctx` tokens (pages reserved, contents whatever the cache holds), runs
warm-up steps, then one instrumented eager decode step, and returns stage ->
milliseconds plus the bytes each stage must move, so every stage can be read
against the measured HBM roofline.
"""
from __future__ import annotations

import time

import torch

from ..utils.stage_timer import StageTimer
from .scheduler import Request, ScheduledSeq, Status


def profile_decode(engine, batch: int, ctx: int, reps: int = 3, graph: bool = False) -> dict:
    """`graph=True` captures the instrumented step in a CUDA graph (the timer's
    events become event-record nodes) and times a replay, so launch overhead of
    the eager path does not leak into the stage times."""
    m = engine.model
    reqs = []
    for _ in range(batch):
        r = Request([1] * ctx, 4)
        engine.kv.open(r.rid, [])
        engine.kv.append(r.rid, [1] * ctx)
        r.status = Status.DECODE
        r.output = [1]
        reqs.append(r)
    res = {}
    try:
        for rep in range(reps + 1):
            sched = [ScheduledSeq(r, [int(torch.randint(0, m.cfg.vocab_size, (1,)))], r.seq_len - 1 + rep, True)
                     for r in reqs]
            T, S, w, n_out = engine._stage(sched, batch)
            timer = StageTimer(enabled=rep == reps)
            m.timer = timer
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if graph and rep == reps:
                g = torch.cuda.CUDAGraph()
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.graph(g, stream=s):
                    m.forward(T, S, w, n_out, True)
                torch.cuda.synchronize()
                for _ in range(2):
                    g.replay()
                torch.cuda.synchronize()
                ev0.record()
                g.replay()
                ev1.record()
                torch.cuda.synchronize()
            else:
                ev0.record()
                m.forward(T, S, w, n_out, True)
                ev1.record()
                torch.cuda.synchronize()
            if rep == reps:
                res = timer.resolve()
                res["_step_ms"] = ev0.elapsed_time(ev1)
                res["_host_ms"] = (time.perf_counter() - t0) * 1e3
    finally:
        m.timer = StageTimer(False)
        for r in reqs:
            engine.kv.free(r.rid)
    return res


def profile_decode_kernels(engine, batch: int, ctx: int, replays: int = 5) -> dict:
    """Per-kernel device time of a captured decode step, from CUPTI activity records
    (torch.profiler) over `replays` graph replays.  Diagnosis only: reported
    throughput always comes from CUDA events without a profiler attached."""
    import torch.profiler as tp
    m = engine.model
    reqs = []
    for _ in range(batch):
        r = Request([1] * ctx, 4)
        engine.kv.open(r.rid, [])
        engine.kv.append(r.rid, [1] * ctx)
        r.status = Status.DECODE
        r.output = [1]
        reqs.append(r)
    try:
        sched = [ScheduledSeq(r, [int(torch.randint(0, m.cfg.vocab_size, (1,)))], r.seq_len - 1, True)
                 for r in reqs]
        T, S, w, n_out = engine._stage(sched, batch)
        m.forward(T, S, w, n_out, True)  # warm-up (workspaces, attributes)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g, stream=s):
            m.forward(T, S, w, n_out, True)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(replays):
            g.replay()
        ev1.record()
        torch.cuda.synchronize()
        step_ms = ev0.elapsed_time(ev1) / replays
        with tp.profile(activities=[tp.ProfilerActivity.CUDA]) as prof:
            for _ in range(replays):
                g.replay()
            torch.cuda.synchronize()
        agg = {}
        seq = [e for e in prof.events() if e.device_type == tp.DeviceType.CUDA]
        seq.sort(key=lambda e: e.time_range.start)
        per = len(seq) // replays
        one = seq[:per]
        timeline = []
        for e in one[40:40 + 60]:  # a few layers past the first ones
            nm = e.name
            short = nm.split("(")[0].replace("void ", "").replace("rkt::", "")
            timeline.append((short[:60], round(e.time_range.elapsed_us(), 1)))
        for e in prof.events():
            if e.device_type == tp.DeviceType.CUDA:
                name = e.name
                for key in ("gemm_kernel", "attn_decode_kernel", "attn_kernel", "sp_land_kernel", "moe_dispatch_sp",
                            "moe_owner_plan_sp", "quantize_rows_list", "qk_rope_kv", "splitk_reduce", "argmax",
                            "embed_kernel", "nccl", "Memcpy", "attn_combine", "elementwise", "reduce"):
                    if key.lower() in name.lower():
                        name = key
                        break
                a = agg.setdefault(name, [0.0, 0])
                a[0] += e.device_time_total / 1e3 / replays if hasattr(e, "device_time_total") else 0.0
                a[1] += 1
        del g
        return {"step_ms": step_ms, "timeline_us": timeline,
                "kernels": {k: {"ms_per_step": round(v[0], 3), "launches_per_step": v[1] // replays}
                            for k, v in sorted(agg.items(), key=lambda kv: -kv[1][0])}}
    finally:
        for r in reqs:
            engine.kv.free(r.rid)


def kernel_breakdown(fn, reps: int = 4, top: int = 25) -> dict:
    """Device time per kernel name over `reps` calls of fn() (CUPTI activity records via
    torch.profiler).  Diagnosis only: reported throughput always comes from CUDA events
    without a profiler attached."""
    import torch.profiler as tp
    torch.cuda.synchronize()
    with tp.profile(activities=[tp.ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
    agg: dict[str, list] = {}
    total = 0.0
    for e in prof.events():
        if e.device_type != tp.DeviceType.CUDA:
            continue
        name = e.name.split("(")[0].replace("void ", "").replace("rkt::", "")
        if "<" in name:
            base, tmpl = name.split("<", 1)
            name = base + "<" + tmpl[:24]
        us = e.time_range.elapsed_us()
        a = agg.setdefault(name[:80], [0.0, 0])
        a[0] += us
        a[1] += 1
        total += us
    rows = sorted(agg.items(), key=lambda kv: -kv[1][0])[:top]
    return {"device_ms_per_call": round(total / 1e3 / reps, 3),
            "kernels": [{"name": k, "ms_per_call": round(v[0] / 1e3 / reps, 3), "launches_per_call": v[1] // reps,
                         "share": round(v[0] / total, 3) if total else 0.0} for k, v in rows]}


def host_overhead(batch: int, spec: int = 0, steps: int = 40, heads=(96, 8), python_stage: bool = False) -> dict:
    """Median host milliseconds per decode step of the scheduler (schedule), the step
    staging (KV slot reservation + packed metadata + block table) and the completion
    (token bookkeeping, speculative rollback) for `batch` decoding sequences -- no GPU:
    the engine's host state runs with CPU metadata buffers.  `python_stage` times the
    Python restatement of the staging instead of the native stager."""
    import types

    from .. import _rt
    from .engine import LLMEngine, StepStats
    from .scheduler import Scheduler, SeqResult
    Hq, Hkv = heads
    T, S, W, O, mpp = max(4096, batch * (spec + 1)), batch, 4096, max(2048, batch * (spec + 1)), 64
    e = LLMEngine.__new__(LLMEngine)
    e.K = spec
    e.model = types.SimpleNamespace(Hq=Hq, Hkv=Hkv, max_tokens=T, max_seqs=S, max_work=W, max_out=O,
                                    block_table=torch.zeros(S, mpp, dtype=torch.int32))
    e.meta_len = 3 * T + 3 * S + 2 * W + 1 + O + S + ((2 * S + 2 * T) if spec else 0)
    e.meta_dev = torch.zeros(e.meta_len, dtype=torch.int32)
    e.meta_host = torch.zeros(e.meta_len, dtype=torch.int32)
    e.bt_host = torch.zeros(S, mpp, dtype=torch.int32)
    e._bind_meta()
    pages = batch * mpp + 1
    e.kv = _rt.KvManager(pages - 1, 64, mpp, False)
    e.ecfg = types.SimpleNamespace(page_size=64)
    e.dummy_page, e.dummy_slot = pages - 1, S
    e.slot_of, e.free_slots = {}, list(range(S - 1, -1, -1))
    e.stats = StepStats()
    e._py_stage = python_stage
    sch = Scheduler(e.kv, batch, 1 << 20, 1 << 20, spec)
    e.sched = sch
    for _ in range(batch):
        r = Request(list(range(30)), 1 << 20)
        e.kv.open(r.rid, [])
        e.kv.append(r.rid, list(range(30)))
        r.status, r.output, r.computed, r.drafts = Status.DECODE, [1], 30, [2] * spec
        sch.running.append(r)
    ts = {"schedule": [], "stage": [], "complete": []}
    for _ in range(steps):
        t0 = time.perf_counter()
        sched = sch.schedule()
        t1 = time.perf_counter()
        e._stage(sched, batch)
        t2 = time.perf_counter()
        res = [SeqResult([5, 6] if spec else [5], (s.start + 2) if spec else None, [3] * spec if spec else None)
               for s in sched]
        t3 = time.perf_counter()
        sch.complete(sched, res, t3)
        t4 = time.perf_counter()
        ts["schedule"].append(t1 - t0)
        ts["stage"].append(t2 - t1)
        ts["complete"].append(t4 - t3)
    out = {k: round(1e3 * sorted(v)[len(v) // 2], 3) for k, v in ts.items()}
    out["total"] = round(sum(out.values()), 3)
    return out


if __name__ == "__main__":
    import json
    import sys
    b = int(sys.argv[1]) if len(sys.argv) > 1 else 64
    k = int(sys.argv[2]) if len(sys.argv) > 2 else 0
    print(json.dumps({"batch": b, "spec": k, "native_ms": host_overhead(b, k),
                      "python_stage_ms": host_overhead(b, k, python_stage=True)}))
