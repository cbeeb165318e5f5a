"""Draft sources for speculative verify steps.

A verify step feeds ``[last, d_1 .. d_K]`` for every decoding sequence and the
device keeps the longest prefix of drafts that matches its own greedy argmax, so
any proposal is safe: drafts only change how many tokens a step emits, never
which.  The engine's default drafts are the MTP head's chain from the previous
step (computed on the device inside the same CUDA graph).  The sources here
replace or complement them from the host:

* ``PromptLookup``  -- n-gram match of the sequence's own suffix against its
  prompt + output (code and retrieval prompts repeat themselves).  The newest
  occurrence with the longest match wins; matching is incremental (an index from
  each ``n_min``-gram to its most recent end positions), so a 32k-token prompt
  costs O(new tokens) per step instead of a rescan.
* ``HistoryBigram`` -- the generated tokens' own last bigram, looked up in the
  generated tokens (the fallback of the reference's bench when nothing else
  proposes).
* ``DraftFile``     -- the continuation of a reference generation (perfect drafts:
  a correctness probe for the acceptance / rollback path).
* ``DraftModel``    -- a separate smaller model on its own engine, batched greedy
  drafting for all decoding sequences once per step.
* ``Chain``         -- first source that proposes anything; short proposals are
  padded with the MTP drafts, then with the last token.

Counterpart of the draft-source selection in the reference's coding bench
(engines/glm5-moe-nvfp4-2b/src/coding_bench_main.cu:590-665: ``--draft-file``,
``ROCKET_PROMPT_LOOKUP`` n-gram 8..3, DFlash2, history bigram).  Every source is a
pure function of the request's tokens, so all ranks propose the same drafts
without exchanging them.
"""
from __future__ import annotations

import json
from collections import deque


class DraftSource:
    """propose(req, K) -> up to K draft tokens (may be empty); release(req) drops state."""

    name = "none"

    def propose(self, req, K: int) -> list[int]:
        return []

    def release(self, req) -> None:
        pass


class MtpDrafts(DraftSource):
    """The MTP head's chain from the previous step (device drafts returned with the step)."""

    name = "mtp"

    def propose(self, req, K):
        return list(req.drafts[:K])


class _Index:
    __slots__ = ("hist", "pos", "n_idx")

    def __init__(self):
        self.hist: list[int] = []
        self.pos: dict = {}   # n_min-gram -> deque of end positions (newest last)
        self.n_idx = 0        # history positions whose n-gram is indexed


class PromptLookup(DraftSource):
    """Longest-suffix n-gram lookup in the sequence's own prompt + output.

    The suffix of length ``n`` (n_max down to n_min) is matched against earlier
    positions; a match ending at position p proposes ``hist[p : p+K]``.  Only matches
    whose whole continuation lies in the history are considered (a match too close
    to the end would propose fewer than K tokens).  Candidates come from an index of
    ``n_min``-grams keeping the ``keep`` most recent end positions each; the longest
    backward extension wins, newest first on ties.
    """

    name = "prompt_lookup"

    def __init__(self, n_max: int = 8, n_min: int = 3, keep: int = 8, min_tokens: int = 1):
        if not 1 <= n_min <= n_max:
            raise ValueError("need 1 <= n_min <= n_max")
        self.n_max, self.n_min, self.keep, self.min_tokens = n_max, n_min, keep, min_tokens
        self._st: dict[int, _Index] = {}

    def _sync(self, req) -> _Index:
        st = self._st.get(req.rid)
        if st is None:
            st = self._st[req.rid] = _Index()
        h = st.hist
        full = len(req.prompt) + len(req.output)
        if len(h) > full:  # the request was rolled back / restarted: rebuild
            st = self._st[req.rid] = _Index()
            h = st.hist
        if len(h) < len(req.prompt):
            h.extend(req.prompt[len(h):])
        if len(h) < full:
            h.extend(req.output[len(h) - len(req.prompt):])
        return st

    def propose(self, req, K):
        st = self._sync(req)
        h, n0 = st.hist, self.n_min
        L = len(h)
        # index n_min-grams ending at p (exclusive) once their continuation h[p:p+K] exists
        upto = L - K
        while st.n_idx < upto:
            p = st.n_idx + 1
            st.n_idx = p
            if p < n0:
                continue
            key = tuple(h[p - n0:p])
            dq = st.pos.get(key)
            if dq is None:
                dq = st.pos[key] = deque(maxlen=self.keep)
            dq.append(p)
        if L < n0:
            return []
        cands = st.pos.get(tuple(h[L - n0:L]))
        if not cands:
            return []
        best, best_n = -1, 0
        for p in reversed(cands):
            n = n0
            while n < self.n_max and p - n - 1 >= 0 and h[p - n - 1] == h[L - n - 1]:
                n += 1
            if n > best_n:
                best, best_n = p, n
                if n == self.n_max:
                    break
        if best < 0:
            return []
        out = h[best:best + K]
        return out if len(out) >= self.min_tokens else []

    def release(self, req):
        self._st.pop(req.rid, None)


class HistoryBigram(DraftSource):
    """Most recent earlier occurrence of the output's last two tokens, in the output."""

    name = "history"

    def propose(self, req, K):
        g = req.output
        if len(g) < 3:
            return []
        a, b = g[-2], g[-1]
        for i in range(len(g) - 3, -1, -1):
            if g[i] == a and g[i + 1] == b:
                return list(g[i + 2:i + 2 + K])
        return []


class DraftFile(DraftSource):
    """Drafts read from a reference generation.

    The file is JSON: a list of token-id lists (request i of the run uses list i, in
    order of first proposal) or an object mapping a request's prompt key (its token
    ids joined by ',') to its continuation.  A request with output length g proposes
    ``ref[g : g+K]``.
    """

    name = "file"

    def __init__(self, path_or_obj):
        obj = path_or_obj
        if isinstance(path_or_obj, str):
            with open(path_or_obj) as f:
                obj = json.load(f)
        if isinstance(obj, dict):
            self.by_prompt = {k: [int(t) for t in v] for k, v in obj.items()}
            self.by_order = None
        elif isinstance(obj, list):
            self.by_order = [[int(t) for t in v] for v in obj]
            self.by_prompt = None
        else:
            raise ValueError("draft file must hold a list of token lists or a prompt -> tokens object")
        self._assigned: dict[int, list[int]] = {}

    @staticmethod
    def prompt_key(prompt) -> str:
        return ",".join(str(int(t)) for t in prompt)

    def _ref(self, req):
        ref = self._assigned.get(req.rid)
        if ref is None:
            if self.by_prompt is not None:
                ref = self.by_prompt.get(self.prompt_key(req.prompt), [])
            else:
                i = len(self._assigned)
                ref = self.by_order[i] if i < len(self.by_order) else []
            self._assigned[req.rid] = ref
        return ref

    def propose(self, req, K):
        g = len(req.output)
        return list(self._ref(req)[g:g + K])

    def release(self, req):
        pass  # keep the assignment: a request's reference stays fixed for the whole run


class DraftModel(DraftSource):
    """A separate (smaller) model drafts K tokens greedily for every decoding sequence.

    Before each target step the engine calls ``prepare`` with its decoding requests and
    this source runs ONE batched greedy generation of K tokens on its own engine over
    all of their contexts (prompt + output); the draft engine's prefix cache keeps the
    full pages of earlier contexts, so each step re-prefills only the tail since the
    last full page plus the newly accepted tokens.  The draft model must share the
    target's vocabulary; under tensor parallelism every rank builds the same draft
    engine and runs it in lockstep, so the drafts agree without an exchange.

    Counterpart of the reference's separate drafter (DFlash2, engines/glm5-moe-nvfp4-2b/
    src/dflash2.h:19-91), as a generic draft model: the DFlash2-specific conditioning on
    target hidden taps is not part of it.
    """

    name = "draft_model"

    def __init__(self, engine):
        if engine.K:
            raise ValueError("the draft engine itself must not speculate")
        self.engine = engine
        self.vocab_size = engine.model.cfg.vocab_size
        self._ready: dict = {}
        self.steps = 0

    def prepare(self, reqs, K: int) -> None:
        from .scheduler import Status
        live = [r for r in reqs if r.status == Status.DECODE]
        self._ready = {}
        if not live:
            return
        lim = self.engine.sched.max_seq_len - K
        ctxs = [(list(r.prompt) + list(r.output))[-lim:] for r in live]
        outs = self.engine.generate(ctxs, K)
        self._ready = {r.rid: o for r, o in zip(live, outs)}
        self.steps += 1

    def propose(self, req, K):
        return list(self._ready.pop(req.rid, []))[:K]


class Chain(DraftSource):
    """The first source with a proposal; padded to K with the MTP drafts, then the last token."""

    def __init__(self, sources):
        self.sources = list(sources)
        self.name = "+".join(s.name for s in self.sources)
        self.hits = {s.name: 0 for s in self.sources}

    def prepare(self, reqs, K: int) -> None:
        """Batched work of the sources before a step's proposals (a draft model's run)."""
        for s in self.sources:
            if hasattr(s, "prepare"):
                s.prepare(reqs, K)

    def propose(self, req, K):
        d: list[int] = []
        for s in self.sources:
            d = s.propose(req, K)
            if d:
                self.hits[s.name] += 1
                break
        if len(d) < K:
            mtp = list(req.drafts)
            d = d + mtp[len(d):K]
        if len(d) < K:
            last = req.output[-1] if req.output else (req.prompt[-1] if req.prompt else 0)
            d = d + [last] * (K - len(d))
        return d[:K]

    def release(self, req):
        for s in self.sources:
            s.release(req)


def wilson_bounds(k: int, n: int, z: float = 1.96) -> tuple[float, float]:
    """Wilson score interval of a binomial rate k / n."""
    if n <= 0:
        return 0.0, 1.0
    p = k / n
    den = 1 + z * z / n
    mid = (p + z * z / (2 * n)) / den
    half = z * ((p * (1 - p) / n + z * z / (4 * n * n)) ** 0.5) / den
    return max(0.0, mid - half), min(1.0, mid + half)


class AdaptiveChain(Chain):
    """A Chain whose host sources are demoted per request while their drafts keep
    failing, so the next source (eventually the MTP drafts) drafts instead.

    Each step's acceptance is attributed to the source that proposed the verified
    drafts (from the request's drafted / accepted counters).  A source is skipped for a
    request once the Wilson upper bound of its per-draft acceptance over its last
    `window` drafted tokens falls below `min_rate`; every `explore_every`-th proposal for
    that request probes it again, and the probe's outcome joins its window (a source
    that recovers is promoted back).  Sources without enough evidence (fewer than
    `min_drafts` drafts) are always tried.  Spec: 'adaptive:prompt_lookup+history+mtp'.

    The counterpart of the reference's adaptive speculation policy (Wilson-bound
    promotion / demotion with exploration: engines/qwen38-flash-next-nvfp4-2b/src/
    qwen38_slab/mtp_policy.py:1-57), applied here to choosing a draft source: a verify
    step's cost does not depend on which source filled its rows.
    """

    def __init__(self, sources, min_rate: float = 0.2, window: int = 64, min_drafts: int = 16,
                 explore_every: int = 32):
        super().__init__(sources)
        self.name = "adaptive:" + self.name
        self.min_rate, self.window, self.min_drafts, self.explore = min_rate, window, min_drafts, explore_every
        self._st: dict = {}      # rid -> {"last": (source idx, drafted0, accepted0) | None, "hist": {i: deque}, "n": int}
        self.skips = {s.name: 0 for s in self.sources}

    def _state(self, req):
        st = self._st.get(req.rid)
        if st is None:
            st = self._st[req.rid] = {"last": None, "hist": {}, "n": 0}
        return st

    def _demoted(self, st, i) -> bool:
        h = st["hist"].get(i)
        if not h:
            return False
        n = sum(d for d, _ in h)
        if n < self.min_drafts:
            return False
        return wilson_bounds(sum(a for _, a in h), n)[1] < self.min_rate

    def propose(self, req, K):
        st = self._state(req)
        if st["last"] is not None:  # attribute the verified step to its proposer
            i, d0, a0 = st["last"]
            dd, da = req.drafted - d0, req.accepted - a0
            if dd > 0:
                h = st["hist"].setdefault(i, deque())
                h.append((dd, da))
                while sum(d for d, _ in h) - h[0][0] >= self.window:
                    h.popleft()
        st["n"] += 1
        explore = self.explore and st["n"] % self.explore == 0
        d: list[int] = []
        who = None
        for i, s in enumerate(self.sources):
            if self._demoted(st, i) and not explore:
                self.skips[s.name] += 1
                continue
            d = s.propose(req, K)
            if d:
                self.hits[s.name] += 1
                who = i
                break
        st["last"] = (who, req.drafted, req.accepted) if who is not None else None
        if len(d) < K:
            d = d + list(req.drafts)[len(d):K]
        if len(d) < K:
            last = req.output[-1] if req.output else (req.prompt[-1] if req.prompt else 0)
            d = d + [last] * (K - len(d))
        return d[:K]

    def release(self, req):
        super().release(req)
        self._st.pop(req.rid, None)


def make_draft_source(spec: str, draft_file: str | None = None, draft_engine=None) -> Chain | None:
    """``spec``: '+'-joined source names in priority order, e.g. 'prompt_lookup+mtp',
    'file', 'history', 'draft_model' (needs `draft_engine`, an LLMEngine of the draft
    model).  'mtp' alone (the engine default) returns None."""
    adaptive = spec.startswith("adaptive:")
    if adaptive:
        spec = spec[len("adaptive:"):]
    names = [s.strip() for s in spec.split("+") if s.strip()]
    if not names or names == ["mtp"]:
        return None
    srcs = []
    for n in names:
        if n == "mtp":
            srcs.append(MtpDrafts())
        elif n in ("prompt_lookup", "lookup", "ngram"):
            srcs.append(PromptLookup())
        elif n == "history":
            srcs.append(HistoryBigram())
        elif n == "file":
            if not draft_file:
                raise ValueError("draft source 'file' needs a draft file")
            srcs.append(DraftFile(draft_file))
        elif n in ("draft_model", "model"):
            if draft_engine is None:
                raise ValueError("draft source 'draft_model' needs a draft engine")
            srcs.append(DraftModel(draft_engine))
        else:
            raise ValueError(f"unknown draft source {n!r}")
    return AdaptiveChain(srcs) if adaptive else Chain(srcs)
