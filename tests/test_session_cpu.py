"""SessionStore logic on the CPU with a fake engine (page caches as CPU tensors): the
disk record and the multi-rank transaction paths restore every cache family (including a
zero-sized V cache as MLA has, DSA index caches, DeltaNet state) bit for bit."""
import types

import pytest
import torch

rt = pytest.importorskip("rocket_b200._rt")


class FakeModel:
    def __init__(self, pages=16, ps=4, mla=False, dn=False):
        g = torch.Generator().manual_seed(0)
        self.page_size, self.dev = ps, torch.device("cpu")
        L = 3
        if mla:
            self.k_cache = torch.randn(L, pages, 1, ps, 32, generator=g).bfloat16()
            self.v_cache = torch.zeros(L, pages, 1, 0, ps, dtype=torch.bfloat16)
        else:
            self.k_cache = torch.randn(L, pages, 2, ps, 8, generator=g).bfloat16()
            self.v_cache = torch.randn(L, pages, 2, 8, ps, generator=g).bfloat16()
        self.ik = torch.randn(L, pages * ps, 16, generator=g).bfloat16()
        self.num_pages = pages
        if dn:
            self.dn_buf = types.SimpleNamespace(state=torch.randn(2, 5, 4, 8, 8, generator=g),
                                                conv_state=torch.randn(2, 5, 3, 24, generator=g).bfloat16())
        self.cfg = types.SimpleNamespace(name="fake", num_layers=L, d_model=8, num_q_heads=2, num_kv_heads=2,
                                         head_dim=8, vocab_size=100)
        self.par = types.SimpleNamespace(tp=1, tp_rank=0)

    def page_caches(self):
        L = self.ik.shape[0]
        return [self.k_cache, self.v_cache, self.ik.view(L, self.num_pages, self.page_size, -1)]


class FakeEngine:
    def __init__(self, **kw):
        from rocket_b200.engine.scheduler import Scheduler
        self.model = FakeModel(**kw)
        self.kv = rt.KvManager(self.model.num_pages, self.model.page_size, 8, False)
        self.hybrid = kw.get("dn", False)
        self.slot_of, self.free_slots = {}, [4, 3, 2, 1, 0]
        self.sched = Scheduler(self.kv, 4, 64, 64, 0)


def _running(eng, prompt, out):
    from rocket_b200.engine.scheduler import Request, Status
    r = Request(list(prompt), 20)
    r.output = list(out)
    eng.kv.open(r.rid, [])
    eng.kv.append(r.rid, r.prompt + r.output[:-1])
    r.computed = len(r.prompt) + len(r.output) - 1
    r.status = Status.DECODE
    eng.slot_of[r.rid] = eng.free_slots.pop()
    return r


@pytest.mark.parametrize("kind", ["gqa", "mla", "hybrid"])
def test_session_round_trip_restores_every_cache(tmp_path, kind):
    from rocket_b200.kv.prefix_store import SessionStore
    from rocket_b200.kv.state_txn import DistributedTxn
    kw = {"mla": kind == "mla", "dn": kind == "hybrid"}
    a = FakeEngine(**kw)
    r = _running(a, [5, 6, 7, 8, 9, 10, 11], [12, 13])
    pages = list(a.kv.pages(r.rid))
    want = [c[:, pages].clone() for c in a.model.page_caches()]
    slot = a.slot_of[r.rid]
    if kind == "hybrid":
        want_state = a.model.dn_buf.state[:, slot].clone()
    for path in ("record", "txn"):
        b = FakeEngine(**kw)
        for c in b.model.page_caches():
            c.zero_()
        if path == "record":
            key = SessionStore(a, str(tmp_path / "rec")).save(r)
            r2 = SessionStore(b, str(tmp_path / "rec")).resume(key)
        else:
            SessionStore(a, str(tmp_path / "rec")).save_txn(r, "s1", DistributedTxn(str(tmp_path / "txn")))
            r2 = SessionStore(b, str(tmp_path / "rec")).resume_txn("s1", DistributedTxn(str(tmp_path / "txn")))
        assert r2.prompt == r.prompt and r2.output == r.output and r2.computed == r.computed
        p2 = list(b.kv.pages(r2.rid))
        for w, c in zip(want, b.model.page_caches()):
            assert torch.equal(c[:, p2], w)
        if kind == "hybrid":
            assert torch.equal(b.model.dn_buf.state[:, b.slot_of[r2.rid]], want_state)
