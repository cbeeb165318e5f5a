"""Serving metrics with bounded label cardinality, rendered in the Prometheus text
exposition format (no client library needed).

Counters: requests, prompt / generated tokens, engine steps, speculative drafts
(drafted / accepted), prefix-cache lookups / hits, graph replays.
Gauges: running / waiting requests, free KV pages.
Histograms (fixed buckets): step milliseconds, TTFT, inter-token latency.

Counterpart of the reference's machine-readable result JSON and OpenTelemetry
stage metrics (engines/glm5-moe-nvfp4-2b/src/coding_bench_main.cu:884-933,
engines/qwen38-flash-next-nvfp4-2b/src/pair_reduce/otel.h:8-51).
"""
from __future__ import annotations

import bisect
import threading

MS_BUCKETS = (1, 2, 5, 10, 20, 50, 100, 200, 500, 1000, 2000, 5000, 10000, 30000)


class Histogram:
    def __init__(self, buckets=MS_BUCKETS):
        self.buckets = tuple(buckets)
        self.counts = [0] * (len(self.buckets) + 1)
        self.sum = 0.0
        self.n = 0

    def observe(self, v: float):
        self.counts[bisect.bisect_left(self.buckets, v)] += 1
        self.sum += v
        self.n += 1


class Metrics:
    COUNTERS = ("requests_total", "prompt_tokens_total", "generated_tokens_total", "steps_total",
                "spec_drafted_total", "spec_accepted_total", "prefix_lookups_total", "prefix_hits_total",
                "graph_replays_total")
    GAUGES = ("running_requests", "waiting_requests", "free_kv_pages")
    HISTS = ("step_ms", "ttft_ms", "itl_ms")

    def __init__(self, prefix: str = "rocket_b200", labels: dict | None = None):
        self.prefix = prefix
        # labels are fixed per engine (rank, fuel): cardinality stays bounded
        self.labels = dict(labels or {})
        self.c = {k: 0 for k in self.COUNTERS}
        self.g = {k: 0.0 for k in self.GAUGES}
        self.h = {k: Histogram() for k in self.HISTS}
        self.lock = threading.Lock()

    def inc(self, name: str, v: int = 1):
        with self.lock:
            self.c[name] += v

    def set(self, name: str, v: float):
        with self.lock:
            self.g[name] = v

    def observe(self, name: str, v: float):
        with self.lock:
            self.h[name].observe(v)

    def _lab(self, extra: dict | None = None) -> str:
        d = dict(self.labels)
        if extra:
            d.update(extra)
        if not d:
            return ""
        return "{" + ",".join(f'{k}="{v}"' for k, v in sorted(d.items())) + "}"

    def render(self) -> str:
        out = []
        p = self.prefix
        with self.lock:
            for k, v in self.c.items():
                out += [f"# TYPE {p}_{k} counter", f"{p}_{k}{self._lab()} {v}"]
            for k, v in self.g.items():
                out += [f"# TYPE {p}_{k} gauge", f"{p}_{k}{self._lab()} {v}"]
            for k, h in self.h.items():
                out.append(f"# TYPE {p}_{k} histogram")
                cum = 0
                for b, n in zip(h.buckets, h.counts):
                    cum += n
                    out.append(f"{p}_{k}_bucket{self._lab({'le': b})} {cum}")
                out.append(f"{p}_{k}_bucket{self._lab({'le': '+Inf'})} {h.n}")
                out.append(f"{p}_{k}_sum{self._lab()} {h.sum}")
                out.append(f"{p}_{k}_count{self._lab()} {h.n}")
        return "\n".join(out) + "\n"
