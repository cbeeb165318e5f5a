"""Host draft sources (prompt lookup, history bigram, draft file) and the scheduler's
verify / rollback loop driven by a simulated greedy model on the CPU."""
import json
import random

import pytest

from rocket_b200.engine.drafts import (Chain, DraftFile, HistoryBigram, MtpDrafts, PromptLookup,
                                       make_draft_source)
from rocket_b200.engine.scheduler import Request, Scheduler, SeqResult


def brute_lookup(h, K, n_min, n_max):
    """Longest suffix match (n_min..n_max) whose continuation h[p:p+K] lies in h; newest wins ties."""
    L = len(h)
    best, best_n = -1, 0
    for p in range(n_min, L - K + 1):
        n = 0
        while n < n_max and p - n - 1 >= 0 and h[p - n - 1] == h[L - n - 1]:
            n += 1
        if n >= n_min and (n > best_n or (n == best_n and p > best)):
            best, best_n = p, n
    return h[best:best + K] if best >= 0 else []


def req(prompt, output=()):
    r = Request(list(prompt), 1000)
    r.output = list(output)
    return r


@pytest.mark.parametrize("seed", range(6))
def test_prompt_lookup_matches_bruteforce(seed):
    rng = random.Random(seed)
    vocab = rng.choice([3, 5, 12])
    K = rng.choice([1, 3, 4])
    pl = PromptLookup(n_max=6, n_min=2, keep=10 ** 9)
    r = req([rng.randrange(vocab) for _ in range(rng.randint(5, 60))])
    for _ in range(40):
        h = r.prompt + r.output
        assert pl.propose(r, K) == brute_lookup(h, K, 2, 6)
        r.output.append(rng.randrange(vocab))   # incremental indexing as the output grows


def test_prompt_lookup_repeated_code():
    body = [7, 8, 9, 10, 11, 12, 13, 14]
    r = req([1, 2] + body + [3, 4] + body[:4])
    assert PromptLookup().propose(r, 3) == [11, 12, 13]
    # rollback (shorter history than indexed) rebuilds the index
    pl = PromptLookup()
    pl.propose(r, 3)
    r2 = req(r.prompt[:6])
    r2.rid = r.rid
    assert pl.propose(r2, 3) == brute_lookup(r2.prompt, 3, 3, 8)


def test_history_bigram_and_file(tmp_path):
    r = req([0], [5, 6, 7, 8, 5, 6])
    assert HistoryBigram().propose(r, 3) == [7, 8, 5]
    p = tmp_path / "d.json"
    p.write_text(json.dumps([[4, 5, 6, 7, 8]]))
    df = DraftFile(str(p))
    r = req([1, 2], [4])
    assert df.propose(r, 3) == [5, 6, 7]
    r.output += [5, 6, 7]
    assert df.propose(r, 3) == [8]
    byp = DraftFile({DraftFile.prompt_key([1, 2]): [9, 9, 9]})
    assert byp.propose(req([1, 2]), 2) == [9, 9]
    assert byp.propose(req([3]), 2) == []


def test_chain_pads_with_mtp_then_last():
    r = req([1, 2, 3], [4])
    r.drafts = [40, 41, 42]
    ch = Chain([HistoryBigram()])
    assert ch.propose(r, 3) == [40, 41, 42]          # nothing proposed: MTP chain
    r.drafts = []
    assert ch.propose(r, 3) == [4, 4, 4]             # no MTP either: last token
    assert make_draft_source("mtp") is None
    assert make_draft_source("prompt_lookup+mtp").name == "prompt_lookup+mtp"
    with pytest.raises(ValueError):
        make_draft_source("file")


# ---------------------------------------------------------------- scheduler loop
rt = pytest.importorskip("rocket_b200._rt")


def true_next(h):
    """The simulated model's greedy token: a periodic function of the last two tokens,
    so generated text repeats itself (prompt lookup has something to find)."""
    return (h[-1] * 7 + h[-2] * 3 + 1) % 23 if len(h) >= 2 else 1


def run(source, K, prompts, max_new):
    kv = rt.KvManager(512, 16, 64, False)
    sch = Scheduler(kv, max_batch=4, token_budget=64, max_seq_len=1024, spec_tokens=K)
    if source is not None:
        sch.draft_hook = lambda r: source.propose(r, K)
    reqs = [Request(list(p), max_new) for p in prompts]
    for r in reqs:
        sch.add(r)
    steps = 0
    while sch.has_work():
        sched = sch.schedule()
        results = []
        for s in sched:
            r = s.req
            h = (r.prompt + r.output)[:s.start] + list(s.tokens)
            if not s.sample:
                results.append(SeqResult([], s.start + len(s.tokens) if s.reserve else None))
                continue
            if s.verify:
                ctx = r.prompt + r.output[:-1]
                emitted = []
                for j in range(len(s.tokens)):
                    t = true_next(ctx + s.tokens[:j + 1])
                    emitted.append(t)
                    if j + 1 >= len(s.tokens) or s.tokens[j + 1] != t:
                        break
                a = len(emitted) - 1
                results.append(SeqResult(emitted, s.start + a + 1, [0] * K))
            else:
                results.append(SeqResult([true_next(h)], s.start + len(s.tokens), [0] * K))
        sch.complete(sched, results, 0.0)
        steps += 1
        assert steps < 10000
    return [r.output for r in reqs], sum(r.accepted for r in reqs) / max(1, sum(r.drafted for r in reqs)), steps


def test_scheduler_exact_under_any_drafts(tmp_path):
    rng = random.Random(0)
    prompts = [[rng.randrange(23) for _ in range(rng.randint(3, 40))] for _ in range(6)]
    ref, _, _ = run(None, 0, prompts, 48)
    # greedy reference continuations for the draft file (perfect drafts)
    f = tmp_path / "ref.json"
    f.write_text(json.dumps(ref))
    for spec in ["mtp", "prompt_lookup+mtp", "history", "file"]:
        src = make_draft_source(spec, str(f)) or MtpDrafts()
        out, acc, steps = run(src, 3, prompts, 48)
        assert out == ref, spec
        if spec == "file":
            assert acc > 0.9   # perfect drafts: nearly every draft accepted
        if spec == "prompt_lookup+mtp":
            assert acc > 0  # the periodic continuation is found in the history


class _FakeDraftEngine:
    """Stands in for a draft LLMEngine: greedy 'model' next = last + 1; records batches."""

    def __init__(self, vocab=1000, max_seq_len=64):
        import types
        self.K = 0
        self.model = types.SimpleNamespace(cfg=types.SimpleNamespace(vocab_size=vocab))
        self.sched = types.SimpleNamespace(max_seq_len=max_seq_len)
        self.batches = []

    def generate(self, ctxs, n):
        self.batches.append([list(c) for c in ctxs])
        return [[(c[-1] + 1 + i) % 1000 for i in range(n)] for c in ctxs]


def test_draft_model_batches_one_run_per_step():
    from rocket_b200.engine.drafts import DraftModel, make_draft_source
    from rocket_b200.engine.scheduler import Request, Status
    fe = _FakeDraftEngine(max_seq_len=40)
    src = make_draft_source("draft_model+history", draft_engine=fe)
    reqs = [Request(list(range(10 * i, 10 * i + 5)), 8) for i in range(3)]
    for r in reqs:
        r.status = Status.DECODE
        r.output = [7]
    pre = Request([1, 2, 3], 4)          # still prefilling: no drafts for it
    src.prepare(reqs + [pre], 3)
    assert len(fe.batches) == 1 and len(fe.batches[0]) == 3
    assert src.propose(reqs[0], 3) == [8, 9, 10]
    assert src.propose(reqs[0], 3) == [7, 7, 7]           # consumed: padded with the last token
    assert src.propose(reqs[1], 2) == [8, 9]
    # contexts longer than the draft engine's limit keep their tail
    long = Request(list(range(100)), 8)
    long.status, long.output = Status.DECODE, [5]
    src.prepare([long], 3)
    assert fe.batches[-1][0] == (list(range(100)) + [5])[-(40 - 3):]
    with pytest.raises(ValueError):
        make_draft_source("draft_model")
    spec_engine = _FakeDraftEngine()
    spec_engine.K = 2
    with pytest.raises(ValueError):
        DraftModel(spec_engine)


def test_adaptive_chain_demotes_a_failing_source_and_explores():
    from rocket_b200.engine.drafts import AdaptiveChain, DraftSource, wilson_bounds
    from rocket_b200.engine.scheduler import Request

    truth = list(range(1000, 2000))

    class Bad(DraftSource):
        name = "bad"

        def propose(self, req, K):
            return [7] * K

    class Good(DraftSource):
        name = "good"

        def propose(self, req, K):
            n = len(req.output)
            return truth[n:n + K]

    src = AdaptiveChain([Bad(), Good()], min_rate=0.3, window=32, min_drafts=12, explore_every=20)
    r = Request([1, 2, 3], 500)
    r.output = [truth[0]]
    used = []
    for step in range(120):
        d = src.propose(r, 3)
        used.append("good" if d == truth[len(r.output):len(r.output) + 3] else "bad")
        a = 0
        for x, y in zip(d, truth[len(r.output):]):
            if x != y:
                break
            a += 1
        r.drafted += 3
        r.accepted += a
        r.output += truth[len(r.output):len(r.output) + a + 1]
    assert used[:4] == ["bad"] * 4                      # no evidence yet: the first source drafts
    assert used[10:].count("bad") <= 110 // 20 + 1      # demoted, probed on exploration ticks only
    assert src.skips["bad"] > 90
    lo, hi = wilson_bounds(0, 12)
    assert lo == 0.0 and hi < 0.3
    src.release(r)
    assert r.rid not in src._st
    from rocket_b200.engine.drafts import make_draft_source
    ch = make_draft_source("adaptive:prompt_lookup+history")
    assert isinstance(ch, AdaptiveChain) and ch.name == "adaptive:prompt_lookup+history"
