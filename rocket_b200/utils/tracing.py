"""Host spans with bounded-cardinality labels, exported as JSON lines or a Chrome trace.

    tr = Tracer(service="rocket_b200", rank=0)
    with tr.span("step", phase="decode", bucket=64):
        ...
    tr.export_chrome("trace.json")        # chrome://tracing / Perfetto
    tr.export_jsonl("spans.jsonl")
    tr.export_otlp_json("spans.otlp.json")  # OpenTelemetry OTLP/JSON

Labels are limited to a fixed key set (rank, phase, bucket, outcome, layer_kind,
stage) and every value is coerced to a short string, so an exporter that turns
labels into metric series cannot blow up (the rule the reference's OpenTelemetry
sink states for its pair-reduce spans: rank, M bucket, dtype, outcome --
engines/qwen38-flash-next-nvfp4-2b/src/pair_reduce/otel.h:8-51).  Spans live in a
bounded ring; a span that raises is recorded with outcome=error and re-raised.
Durations are host wall time; device time comes from the stage timer.
"""
from __future__ import annotations

import json
import os
import threading
import time
from collections import deque

LABEL_KEYS = ("rank", "phase", "bucket", "outcome", "layer_kind", "stage", "dtype")


class _Span:
    __slots__ = ("tr", "name", "labels", "t0")

    def __init__(self, tr, name, labels):
        self.tr, self.name, self.labels = tr, name, labels

    def __enter__(self):
        self.t0 = time.perf_counter_ns()
        return self

    def __exit__(self, et, ev, tb):
        t1 = time.perf_counter_ns()
        lab = dict(self.labels)
        lab.setdefault("outcome", "error" if et is not None else "ok")
        self.tr._record(self.name, lab, self.t0, t1 - self.t0)
        return False


class Tracer:
    def __init__(self, service: str = "rocket_b200", rank: int = 0, capacity: int = 100_000):
        self.service = service
        self.rank = rank
        self.spans: deque = deque(maxlen=capacity)
        self.dropped = 0
        self._lock = threading.Lock()

    @staticmethod
    def _labels(kw) -> dict:
        bad = set(kw) - set(LABEL_KEYS)
        if bad:
            raise ValueError(f"span labels {sorted(bad)} are not in the bounded label set {LABEL_KEYS}")
        return {k: str(v)[:32] for k, v in kw.items()}

    def span(self, name: str, **labels) -> _Span:
        lab = self._labels(labels)
        lab.setdefault("rank", str(self.rank))
        return _Span(self, name, lab)

    def _record(self, name, labels, t0_ns, dur_ns):
        with self._lock:
            if len(self.spans) == self.spans.maxlen:
                self.dropped += 1
            self.spans.append((name, labels, t0_ns, dur_ns))

    def summary(self) -> dict:
        """Per (name, phase) count / total / max milliseconds."""
        out: dict = {}
        for name, lab, _, d in list(self.spans):
            key = f"{name}|{lab.get('phase', '')}"
            e = out.setdefault(key, {"count": 0, "total_ms": 0.0, "max_ms": 0.0})
            e["count"] += 1
            e["total_ms"] += d / 1e6
            e["max_ms"] = max(e["max_ms"], d / 1e6)
        return out

    def export_jsonl(self, path: str):
        with open(path, "w") as f:
            for name, lab, t0, d in list(self.spans):
                f.write(json.dumps({"service": self.service, "name": name, "labels": lab, "start_ns": t0,
                                    "duration_ns": d}) + "\n")

    def export_otlp_json(self, path: str):
        """OpenTelemetry OTLP/JSON (resourceSpans) for an OTel collector's file receiver or
        any OTLP/JSON importer; span times are converted to the epoch clock."""
        import hashlib
        import random
        off = time.time_ns() - time.perf_counter_ns()
        trace_id = hashlib.sha256(f"{self.service}{self.rank}{off}".encode()).hexdigest()[:32]
        rng = random.Random(off)
        spans = []
        for name, lab, t0, d in list(self.spans):
            spans.append({
                "traceId": trace_id, "spanId": "%016x" % rng.getrandbits(64), "name": name, "kind": 1,
                "startTimeUnixNano": str(t0 + off), "endTimeUnixNano": str(t0 + d + off),
                "attributes": [{"key": k, "value": {"stringValue": v}} for k, v in sorted(lab.items())],
                "status": {"code": 2 if lab.get("outcome") == "error" else 1},
            })
        doc = {"resourceSpans": [{
            "resource": {"attributes": [{"key": "service.name", "value": {"stringValue": self.service}},
                                        {"key": "rank", "value": {"intValue": str(self.rank)}}]},
            "scopeSpans": [{"scope": {"name": "rocket_b200"}, "spans": spans}]}]}
        with open(path, "w") as f:
            json.dump(doc, f)

    def export_chrome(self, path: str):
        ev = [{"name": name, "ph": "X", "ts": t0 / 1e3, "dur": d / 1e3, "pid": int(lab.get("rank", 0)),
               "tid": os.getpid(), "args": lab} for name, lab, t0, d in list(self.spans)]
        with open(path, "w") as f:
            json.dump({"traceEvents": ev, "displayTimeUnit": "ms"}, f)


class NullTracer:
    """Disabled tracer: spans cost one attribute lookup."""

    class _N:
        def __enter__(self):
            return self

        def __exit__(self, *a):
            return False

    _n = _N()

    def span(self, name, **labels):
        return self._n

    def summary(self):
        return {}


NULL_TRACER = NullTracer()
