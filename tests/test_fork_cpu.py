"""Engine request bookkeeping on CPU (an engine shell with CPU page caches and recurrent
state): fork (shared full pages, a copied boundary page, copied DeltaNet state and
drafts, refusals), detach / attach / drop, and the parsing of speculative step results."""
import types

import pytest
import torch

rt = pytest.importorskip("rocket_b200._rt")

PS = 16


def _shell(hybrid=False, pages=32, S=4, K=0):
    from rocket_b200.engine.engine import LLMEngine
    from rocket_b200.engine.scheduler import Scheduler
    from rocket_b200.utils.metrics import Metrics
    e = LLMEngine.__new__(LLMEngine)
    e.K = K
    e.kv = rt.KvManager(pages - 1, PS, 16, False)
    k = torch.randn(3, pages, PS, 8)
    v = torch.randn(3, pages, PS, 8)
    e.model = types.SimpleNamespace(page_caches=lambda: [k, v], dn_buf=types.SimpleNamespace(
        state=torch.randn(2, S + 1, 4, 4), conv_state=torch.randn(2, S + 1, 3, 6)))
    e.hybrid = hybrid
    e.sched = Scheduler(e.kv, S, 256, 200, K)
    e.slot_of, e.free_slots = {}, list(range(S - 1, -1, -1))
    e.metrics = Metrics()
    return e, k, v


def _running(e, n_tokens, out=(7, 8)):
    from rocket_b200.engine.scheduler import Request, Status
    r = Request(list(range(n_tokens)), 10)
    r.output = list(out)
    e.kv.open(r.rid, [])
    e.kv.append(r.rid, r.prompt + r.output[:-1])
    r.computed = n_tokens + len(out) - 1
    r.status = Status.DECODE
    r.drafts = [1, 2, 3]
    e.slot_of[r.rid] = e.free_slots.pop()
    e.sched.running.append(r)
    return r


@pytest.mark.parametrize("hybrid", [False, True])
def test_fork_shares_full_pages_and_copies_the_boundary(hybrid):
    e, k, v = _shell(hybrid)
    p = _running(e, 37)               # 38 tokens of KV: 2 full pages + 6 on the boundary page
    c = e.fork(p, 5)
    pp, cp = list(e.kv.pages(p.rid)), list(e.kv.pages(c.rid))
    assert pp[:2] == cp[:2] and pp[2] != cp[2]
    for t in (k, v):
        assert torch.equal(t[:, cp[2]], t[:, pp[2]])
    assert e.kv.length(c.rid) == e.kv.length(p.rid) == p.computed == c.computed
    assert c.prompt == p.prompt and c.output == p.output and c.drafts == p.drafts
    assert c.max_new_tokens == len(p.output) + 5 and c in e.sched.running
    sp, sc = e.slot_of[p.rid], e.slot_of[c.rid]
    assert sp != sc
    b = e.model.dn_buf
    assert torch.equal(b.state[:, sc], b.state[:, sp]) == hybrid
    # both extend independently
    e.kv.append(p.rid, [1])
    e.kv.append(c.rid, [2])
    assert list(e.kv.pages(p.rid))[:3] == pp[:3] and list(e.kv.pages(c.rid))[:3] == cp[:3]


def test_fork_on_a_page_boundary_copies_nothing():
    e, k, v = _shell()
    p = _running(e, 31)               # exactly 32 tokens = 2 full pages
    c = e.fork(p, 3)
    assert list(e.kv.pages(c.rid)) == list(e.kv.pages(p.rid))


def test_fork_refusals():
    from rocket_b200.engine.scheduler import Request
    e, _, _ = _shell(S=2)
    p = _running(e, 20)
    with pytest.raises(ValueError):
        e.fork(Request([1, 2], 3), 3)          # not running
    with pytest.raises(ValueError):
        e.fork(p, 500)                         # past max_seq_len
    e.fork(p, 3)
    with pytest.raises(RuntimeError):
        e.fork(p, 3)                           # batch full


@pytest.mark.parametrize("hybrid", [False, True])
def test_detach_parks_state_and_attach_restores_it(hybrid):
    e, k, v = _shell(hybrid)
    e.drafts = None
    p = _running(e, 37)
    pages = list(e.kv.pages(p.rid))
    slot = e.slot_of[p.rid]
    b = e.model.dn_buf
    st0, cs0 = b.state[:, slot].clone(), b.conv_state[:, slot].clone()
    d = e.detach(p)
    assert p not in e.sched.running and p.rid not in e.slot_of and slot in e.free_slots
    assert list(e.kv.pages(p.rid)) == pages                 # KV stays on the device
    assert (d.state is not None) == hybrid
    b.state[:, slot].zero_()                                # the slot is reused meanwhile
    b.conv_state[:, slot].zero_()
    e.attach(d)
    s2 = e.slot_of[p.rid]
    assert p in e.sched.running and list(e.kv.pages(p.rid)) == pages
    if hybrid:
        assert torch.equal(b.state[:, s2], st0) and torch.equal(b.conv_state[:, s2], cs0)
    d2 = e.detach(p)
    e.drop(d2)
    assert p.status.name == "FINISHED"
    with pytest.raises(ValueError):
        e.detach(p)


@pytest.mark.parametrize("has_mtp", [True, False])
def test_step_results_carry_drafts_only_with_an_mtp_head(has_mtp):
    """A verify step's packed outputs: emitted tokens (accepted drafts + bonus), the
    committed KV length, and next drafts from the MTP head -- none without one."""
    import numpy as np

    from rocket_b200.engine.engine import LLMEngine, StepStats
    from rocket_b200.engine.scheduler import Request, ScheduledSeq
    K, S, O = 3, 2, 8
    e = LLMEngine.__new__(LLMEngine)
    e.K = K
    e.model = types.SimpleNamespace(max_out=O, max_seqs=S, has_mtp=has_mtp)
    e.stats = StepStats()
    r0, r1 = Request([1, 2], 9), Request([3, 4], 9)
    sched = [ScheduledSeq(r0, [5, 6, 7, 8], 10, True, verify=True), ScheduledSeq(r1, [9, 1, 1, 1], 20, True, verify=True)]
    res = np.zeros(O + S + K * S, dtype=np.int64)
    res[:8] = [50, 51, 52, 53, 60, 61, 62, 63]   # target argmax of every verify row
    res[O:O + S] = [2, 0]                         # accepted drafts per sequence
    res[O + S:] = [70, 80, 71, 81, 72, 82]        # next drafts [K][S]
    out = e._results(sched, res, S)
    assert out[0].tokens == [50, 51, 52] and out[0].kv_len == 13
    assert out[1].tokens == [60] and out[1].kv_len == 21
    assert out[0].drafts == ([70, 71, 72] if has_mtp else []) and out[1].drafts == ([80, 81, 82] if has_mtp else [])
