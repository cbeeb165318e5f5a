"""Synthetic serving workloads and an open-loop driver.

    wl = poisson_workload(n=256, rate=None, prompt=(1024, 32768), mean_out=512, vocab=151552)
    res = run_open_loop(engine, wl)

A workload is a list of ``Arrival(t, prompt, max_new_tokens)``: arrival times
from a Poisson process at `rate` requests/s (``rate=None`` saturates the box:
every request arrives at t=0 and the scheduler's admission control -- free KV
pages and the batch limit -- sets the concurrency), prompt lengths uniform in
[lo, hi], output lengths geometric with the given mean, prompt ids uniform
random (prefix-free).  The driver adds each request when the wall clock passes
its arrival time and steps the engine until everything finished (or a time
limit), then reports throughput and latency percentiles.

Counterpart of the reference's workload generators (scripts/scheduler/
agent-workload.py, scripts/baseline/openai-forked-prefix.py), here for the
long-context continuous-batching sweep.
"""
from __future__ import annotations

import math
import random
import time
from dataclasses import dataclass


@dataclass
class Arrival:
    t: float
    prompt: list
    max_new_tokens: int


def geometric(rng: random.Random, mean: float) -> int:
    """Geometric on {1, 2, ...} with the given mean."""
    p = 1.0 / max(mean, 1.0)
    u = 1.0 - rng.random()
    return max(1, int(math.ceil(math.log(u) / math.log(1.0 - p)))) if p < 1 else 1


def poisson_workload(n: int, rate: float | None, prompt: tuple[int, int], mean_out: float, vocab: int,
                     seed: int = 0, max_out: int | None = None) -> list[Arrival]:
    rng = random.Random(seed)
    t = 0.0
    out = []
    for _ in range(n):
        if rate:
            t += rng.expovariate(rate)
        L = rng.randint(prompt[0], prompt[1])
        o = geometric(rng, mean_out)
        if max_out:
            o = min(o, max_out)
        out.append(Arrival(t, [rng.randrange(vocab) for _ in range(L)], o))
    return out


def _pct(a, q):
    if not a:
        return None
    a = sorted(a)
    return a[min(len(a) - 1, int(q * len(a)))]


def run_open_loop(engine, workload: list[Arrival], time_limit_s: float | None = None) -> dict:
    pending = sorted(workload, key=lambda a: a.t)
    reqs = []
    t0 = time.perf_counter()
    i = 0
    out0 = 0
    while i < len(pending) or engine.sched.has_work():
        now = time.perf_counter() - t0
        while i < len(pending) and pending[i].t <= now:
            r = engine.add_request(pending[i].prompt, pending[i].max_new_tokens)
            r.arrival = t0 + pending[i].t
            reqs.append(r)
            i += 1
        if engine.sched.has_work():
            engine.step()
        elif i < len(pending):
            time.sleep(min(0.01, max(0.0, pending[i].t - now)))
        if time_limit_s is not None and now > time_limit_s:
            break
    wall = time.perf_counter() - t0
    done = [r for r in reqs if r.t_done is not None]
    out_tok = sum(len(r.output) for r in reqs) - out0
    ttft = [(r.t_first - r.arrival) * 1e3 for r in reqs if r.t_first]
    itl = []
    for r in reqs:
        itl += [(b - a) * 1e3 for a, b in zip(r.t_tokens, r.t_tokens[1:])]
    res = {
        "requests": len(reqs), "completed": len(done), "wall_s": round(wall, 3),
        "output_tokens": out_tok, "output_tok_s": round(out_tok / wall, 2) if wall else None,
        "prompt_tokens": sum(len(r.prompt) for r in reqs),
        "ttft_ms_p50": _pct(ttft, 0.5), "ttft_ms_p95": _pct(ttft, 0.95),
        "itl_ms_p50": _pct(itl, 0.5), "itl_ms_p95": _pct(itl, 0.95),
        "max_running": None,
    }
    if engine.K:
        res["spec"] = engine.spec_summary(reqs)
    return res
