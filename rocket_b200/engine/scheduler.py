"""Continuous-batching scheduler with chunked prefill.

Every engine step runs all running decode sequences plus as many prefill
chunks as the per-step token budget allows (decode first, so inter-token
latency of running requests is protected), admitting waiting requests while
KV pages last.  A sequence whose prompt is fully prefilled samples its first
token in the same step as its last chunk.

Reference counterparts: the coding-bench admission / chunked prefill / slot
replacement loop (engines/glm5-moe-nvfp4-2b/src/coding_bench_main.cu:357-489,
743-779; chunk 32 + tail 32) -- here the chunk size is a token budget shared by
all prefilling requests, and replacement is continuous.
"""
from __future__ import annotations

import itertools
import time
from dataclasses import dataclass, field
from enum import Enum


class Status(Enum):
    WAITING = 0
    PREFILL = 1
    DECODE = 2
    FINISHED = 3


_ids = itertools.count()


@dataclass
class Request:
    prompt: list
    max_new_tokens: int = 128
    stop_ids: tuple = ()
    arrival: float = field(default_factory=time.perf_counter)
    rid: int = field(default_factory=lambda: next(_ids))
    status: Status = Status.WAITING
    output: list = field(default_factory=list)
    computed: int = 0          # tokens whose KV is written
    cached: int = 0            # tokens reused from the prefix cache
    t_first: float | None = None
    t_tokens: list = field(default_factory=list)
    t_done: float | None = None
    drafts: list = field(default_factory=list)   # speculative tokens proposed for the next step
    drafted: int = 0           # drafts verified so far
    accepted: int = 0          # drafts accepted so far

    @property
    def seq_len(self) -> int:
        return len(self.prompt) + len(self.output)

    def finished(self) -> bool:
        if len(self.output) >= self.max_new_tokens:
            return True
        return bool(self.output) and self.output[-1] in self.stop_ids


@dataclass
class ScheduledSeq:
    req: Request
    tokens: list          # tokens fed this step
    start: int            # position of tokens[0]
    sample: bool          # produces a token this step
    verify: bool = False  # tokens = [last token, drafts...]: a speculative verify
    reserve: int = 0      # extra KV positions reserved past the tokens (draft-pass writes)


@dataclass
class SeqResult:
    tokens: list                      # tokens emitted by the step (empty if it did not sample)
    kv_len: int | None = None         # committed KV length (speculative steps roll back past it)
    drafts: list | None = None        # next step's drafts


class Scheduler:
    def __init__(self, kv, max_batch: int, token_budget: int, max_seq_len: int, spec_tokens: int = 0):
        self.kv = kv
        self.K = spec_tokens
        self.max_batch = max_batch
        self.token_budget = token_budget
        self.max_seq_len = max_seq_len
        self.waiting: list[Request] = []
        self.running: list[Request] = []
        # optional override of the drafts a verify feeds (request -> K tokens); tests use it
        # to feed known continuations
        self.draft_hook = None
        # drafts a verify feeds this step (None: spec_tokens); adaptive depth sets it per step
        self.verify_width: int | None = None
        # lower KV tier hooks (kv/prefix_store.py): before a prompt opens / after it is sealed
        self.before_open = None
        self.after_commit = None

    def add(self, req: Request):
        if len(req.prompt) + req.max_new_tokens > self.max_seq_len:
            raise ValueError(f"request needs {len(req.prompt) + req.max_new_tokens} tokens > max_seq_len "
                             f"{self.max_seq_len}")
        self.waiting.append(req)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def schedule(self) -> list[ScheduledSeq]:
        out: list[ScheduledSeq] = []
        budget = self.token_budget
        # 1) decode: every running sequence past its prompt feeds its last token (plus its
        #    drafts under speculation: [last, d_1..d_K] are verified in one pass)
        K = self.K
        for r in self.running:
            if r.status == Status.DECODE and budget > 0:
                drafts = (self.draft_hook(r) if self.draft_hook else r.drafts) if K else []
                if K:  # exactly this step's verify width (graph buckets need uniform rows)
                    W = K if self.verify_width is None else self.verify_width
                    drafts = (list(drafts) + [r.output[-1]] * W)[:W]
                toks = [r.output[-1]] + list(drafts)
                reserve = K - 1 if K else 0
                if not self.kv.can_append(r.rid, len(toks) + reserve):
                    continue  # out of pages: skip this step (pages free as others finish)
                out.append(ScheduledSeq(r, toks, r.seq_len - 1, True, verify=bool(K), reserve=reserve))
                budget -= len(toks)
        # 2) continue prefills
        for r in self.running:
            if r.status == Status.PREFILL and budget > 0:
                out.append(self._chunk(r, budget))
                budget -= len(out[-1].tokens)
        # 3) admit
        while self.waiting and budget > 0 and len(self.running) < self.max_batch:
            r = self.waiting[0]
            if self.before_open is not None:
                self.before_open(r.prompt)
            cached = self.kv.open(r.rid, list(r.prompt))
            need = self.kv.pages_needed(r.rid, len(r.prompt) - cached + r.max_new_tokens + 2 * self.K)
            if need > self.kv.num_free_pages():
                self.kv.free(r.rid)
                break
            self.waiting.pop(0)
            r.cached = r.computed = cached
            r.status = Status.PREFILL
            self.running.append(r)
            out.append(self._chunk(r, budget))
            budget -= len(out[-1].tokens)
        return [s for s in out if s.tokens]

    def _chunk(self, r: Request, budget: int) -> ScheduledSeq:
        n = min(budget, len(r.prompt) - r.computed)
        toks = r.prompt[r.computed:r.computed + n]
        done = r.computed + n == len(r.prompt)
        return ScheduledSeq(r, toks, r.computed, done, reserve=(self.K - 1 if (done and self.K) else 0))

    def complete(self, sched: list[ScheduledSeq], results: list[SeqResult], now: float):
        """Apply one step's results: advance prefills, append sampled tokens, roll the
        KV of speculative sequences back to what was accepted, retire finished requests."""
        for s, res in zip(sched, results):
            r = s.req
            r.computed = s.start + len(s.tokens)
            if res.kv_len is not None:
                r.computed = res.kv_len
                ops = self.kv.truncate(r.rid, res.kv_len)
                if ops:
                    raise RuntimeError("speculative rollback would copy a shared page")
            if s.verify:
                r.drafted += len(s.tokens) - 1
                r.accepted += len(res.tokens) - 1
            if res.drafts is not None:
                r.drafts = list(res.drafts)
            for tok in res.tokens:
                if r.finished():
                    break
                r.output.append(int(tok))
                r.t_tokens.append(now)
                if r.t_first is None:
                    r.t_first = now
                if r.status == Status.PREFILL:
                    r.status = Status.DECODE
                    self.kv.commit_prefix(r.rid)
                    if self.after_commit is not None:
                        self.after_commit(r.rid)
        done = [r for r in self.running if r.status == Status.DECODE and r.finished()]
        for r in done:
            r.status = Status.FINISHED
            r.t_done = now
            self.kv.free(r.rid)
            self.running.remove(r)
        return done
