"""Native step staging (C++) against a Python restatement of the engine's metadata
semantics: random batches of prefill chunks, decode rows and speculative verify rows,
padded to graph buckets, with two independent KV managers driven identically."""
import random

import numpy as np
import pytest

rt = pytest.importorskip("rocket_b200._rt")

PS = 16


def layout(T, S, W, O, K):
    fields = [("ids", T), ("pos", T), ("slots", T), ("q_start", S), ("q_len", S), ("kv_len", S),
              ("w_seq", W), ("w_tok0", W), ("num_work", 1), ("out_rows", O), ("state_slot", S)]
    if K:
        fields += [("verify", S), ("sample", S), ("out_idx", T), ("next_tok", T)]
    off, o = {}, 0
    for name, n in fields:
        off[name] = (o, n)
        o += n
    return off, o


def stage_py(kv, items, B, K, tpb, dummy_page, dummy_slot, off, meta, bt):
    v = lambda name: meta[off[name][0]:off[name][0] + off[name][1]]
    ids, pos, slots, qs, ql, kl = v("ids"), v("pos"), v("slots"), v("q_start"), v("q_len"), v("kv_len")
    ws, wt, orow, sslot = v("w_seq"), v("w_tok0"), v("out_rows"), v("state_slot")
    if K:
        ver, smp, oidx, ntok = v("verify"), v("sample"), v("out_idx"), v("next_tok")
    t = w = n_out = 0
    seq_ids = []
    for i, (rid, toks, start, sample, verify, reserve, slot, nxt) in enumerate(items):
        k = len(toks)
        sl = kv.append(rid, toks + [0] * reserve)
        ids[t:t + k] = toks
        pos[t:t + k] = np.arange(start, start + k)
        slots[t:t + k] = sl[:k]
        qs[i], ql[i], kl[i] = t, k, start + k
        sslot[i] = slot
        for t0 in range(0, k, tpb):
            ws[w], wt[w] = i, t0
            w += 1
        if K:
            ver[i], smp[i] = verify, sample
            oidx[t:t + k] = -1
            if verify:
                orow[n_out:n_out + k] = np.arange(t, t + k)
                oidx[t:t + k] = np.arange(n_out, n_out + k)
                ntok[t:t + k] = -1
                n_out += k
            else:
                ntok[t:t + len(nxt)] = nxt[:k]
                ntok[t + len(nxt):t + k] = -1
                if sample:
                    orow[n_out] = t + k - 1
                    oidx[t + k - 1] = n_out
                    n_out += 1
        elif sample:
            orow[n_out] = t + k - 1
            n_out += 1
        seq_ids.append(rid)
        t += k
    if seq_ids:
        kv.block_table(seq_ids, bt[:len(items)])
    rows = K + 1 if K else 1
    for i in range(len(items), B):
        ids[t:t + rows] = 0
        pos[t:t + rows] = np.arange(rows)
        slots[t:t + rows] = dummy_page * PS + np.arange(rows)
        qs[i], ql[i], kl[i] = t, rows, rows
        sslot[i] = dummy_slot
        for t0 in range(0, rows, tpb):
            ws[w], wt[w] = i, t0
            w += 1
        orow[n_out:n_out + rows] = np.arange(t, t + rows)
        if K:
            ver[i], smp[i] = 1, 1
            oidx[t:t + rows] = np.arange(n_out, n_out + rows)
            ntok[t:t + rows] = -1
        n_out += rows
        bt[i, 0] = dummy_page
        t += rows
    meta[off["num_work"][0]] = w
    return t, B, w, n_out


@pytest.mark.parametrize("seed", range(30))
def test_native_stager_matches_python(seed):
    rng = random.Random(seed)
    K = rng.choice([0, 0, 3, 2])
    tpb = rng.choice([4, 16, 32])
    T, S, W, O = 512, 16, 512, 256
    off, size = layout(T, S, W, O, K)
    kv_a, kv_b = rt.KvManager(200, PS, 40, False), rt.KvManager(200, PS, 40, False)
    rids = []
    for r in range(rng.randint(1, 8)):
        n0 = rng.randint(0, 40)
        for kv in (kv_a, kv_b):
            kv.open(r, [])
            kv.append(r, list(range(n0)))
        rids.append((r, n0))
    items = []
    for r, n0 in rids:
        kind = rng.choice(["prefill", "decode"])
        if kind == "decode":
            k = K + 1 if K else 1
            items.append((r, [rng.randrange(99) for _ in range(k)], n0, 1, int(bool(K)), K - 1 if K else 0,
                          rng.randrange(8), []))
        else:
            k = rng.randint(1, 30)
            done = rng.random() < 0.5
            nxt = [rng.randrange(99) for _ in range(k if not done else k - 1)]
            items.append((r, [rng.randrange(99) for _ in range(k)], n0, int(done), 0,
                          (K - 1 if (done and K) else 0), rng.randrange(8), nxt))
    B = len(items) + rng.choice([0, 0, 1, 3])
    meta_a = np.full(size, -7, dtype=np.int32)
    meta_b = meta_a.copy()
    bt_a = np.full((S, 40), -5, dtype=np.int32)
    bt_b = bt_a.copy()
    ra = stage_py(kv_a, items, B, K, tpb, 199, 9, off, meta_a, bt_a)
    rb = rt.stage_step(kv_b, items, B, K, tpb, PS, 199, 9, off, meta_b, bt_b)
    assert tuple(rb) == ra
    assert np.array_equal(meta_a, meta_b)
    assert np.array_equal(bt_a, bt_b)
    for r, _ in rids:
        assert list(kv_a.pages(r)) == list(kv_b.pages(r)) and kv_a.length(r) == kv_b.length(r)


def test_native_stager_refuses_overflow_without_side_effects():
    off, size = layout(8, 2, 8, 8, 0)
    kv = rt.KvManager(10, PS, 8, False)
    kv.open(0, [])
    meta = np.zeros(size, dtype=np.int32)
    bt = np.zeros((2, 8), dtype=np.int32)
    with pytest.raises(Exception):
        rt.stage_step(kv, [(0, list(range(9)), 0, 1, 0, 0, 0, [])], 1, 0, 4, PS, 9, 0, off, meta, bt)
    assert kv.length(0) == 0 and not meta.any()


def _shell_engine(K, Hq=8, Hkv=2, T=256, S=8, W=256, O=128, pages=64, mpp=16):
    """An LLMEngine with only the attributes `_stage` touches (no model, no device)."""
    import types

    import torch

    from rocket_b200.engine.engine import LLMEngine, StepStats
    e = LLMEngine.__new__(LLMEngine)
    e.K = K
    e.model = types.SimpleNamespace(Hq=Hq, Hkv=Hkv, max_tokens=T, max_seqs=S, max_work=W, max_out=O,
                                    block_table=torch.zeros(S, mpp, dtype=torch.int32))
    e.meta_len = 3 * T + 3 * S + 2 * W + 1 + O + S + ((2 * S + 2 * T) if K else 0)
    e.meta_dev = torch.zeros(e.meta_len, dtype=torch.int32)
    e.meta_host = torch.zeros(e.meta_len, dtype=torch.int32)
    e.bt_host = torch.zeros(S, mpp, dtype=torch.int32)
    e._bind_meta()
    e.kv = rt.KvManager(pages - 1, PS, mpp, False)
    e.ecfg = types.SimpleNamespace(page_size=PS)
    e.dummy_page, e.dummy_slot = pages - 1, S
    e.slot_of, e.free_slots = {}, list(range(S - 1, -1, -1))
    e.stats = StepStats()
    return e


@pytest.mark.parametrize("K", [0, 3])
def test_engine_stage_native_equals_python_path(K):
    """Both `_stage` paths of the engine on the same schedule: metadata, block table,
    recurrent-state slots and KV reservations agree."""
    import torch

    from rocket_b200.engine.scheduler import Request, ScheduledSeq
    rng = random.Random(K)
    outs = []
    for py in (True, False):
        e = _shell_engine(K)
        e._py_stage = py
        reqs = [Request([rng.randrange(50) for _ in range(20 + 7 * i)], 8, rid=100 + i) for i in range(3)]
        rng.seed(K)
        for r in reqs:
            e.kv.open(r.rid, [])
        steps = []
        # step 1: chunked prefill of all three (the second finishes its prompt)
        sched = [ScheduledSeq(reqs[0], reqs[0].prompt[:16], 0, False),
                 ScheduledSeq(reqs[1], reqs[1].prompt, 0, True, reserve=K - 1 if K else 0),
                 ScheduledSeq(reqs[2], reqs[2].prompt[:9], 0, False)]
        steps.append((e._stage(sched), e.meta_dev.clone(), e.model.block_table.clone()))
        # step 2: a decode / verify row padded to a bucket of 4
        k = K + 1 if K else 1
        sched = [ScheduledSeq(reqs[1], [5] * k, len(reqs[1].prompt), True, verify=bool(K),
                              reserve=K - 1 if K else 0)]
        steps.append((e._stage(sched, 4), e.meta_dev.clone(), e.model.block_table[:4].clone()))
        outs.append((steps, dict(e.slot_of), [list(e.kv.pages(r.rid)) for r in reqs], e.stats.h2d_bytes))
    (sa, slot_a, pages_a, h_a), (sb, slot_b, pages_b, h_b) = outs
    for (ra, ma, ba), (rb, mb, bb) in zip(sa, sb):
        assert tuple(ra) == tuple(rb)
        assert torch.equal(ma, mb) and torch.equal(ba, bb)
    assert slot_a == slot_b and pages_a == pages_b and h_a == h_b


def test_stager_refuses_arrays_it_would_have_to_copy():
    off, size = layout(8, 2, 8, 8, 0)
    kv = rt.KvManager(10, PS, 8, False)
    kv.open(0, [])
    bt = np.zeros((2, 8), dtype=np.int32)
    for meta in (np.zeros(size, dtype=np.int64), np.zeros(2 * size, dtype=np.int32)[::2]):
        with pytest.raises(Exception):
            rt.stage_step(kv, [(0, [1], 0, 1, 0, 0, 0, [])], 1, 0, 4, PS, 9, 0, off, meta, bt)
    assert kv.length(0) == 0
