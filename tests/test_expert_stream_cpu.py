"""Streamed routed experts on the host side: the native LRU slot cache against a
Python model of it, and the streamer's slot fills and id rewriting on CPU tensors."""
import random

import pytest
import torch

rt = pytest.importorskip("rocket_b200._rt")


class _PyCache:
    """Reference model: resident experts first, then free slots, then least recently used."""

    def __init__(self, E, S):
        self.slot_of, self.expert_in, self.last = [-1] * E, [-1] * S, [0] * S
        self.tick = 0

    def plan(self, needed):
        needed = sorted(set(needed))
        res = [e for e in needed if self.slot_of[e] >= 0]
        miss = [e for e in needed if self.slot_of[e] < 0]
        self.tick += 1
        out, mi, first = [], 0, True
        while first or mi < len(miss):
            remap, loads, pinned, used = [-1] * len(self.slot_of), [], set(), 0
            if first:
                for e in res:
                    s = self.slot_of[e]
                    pinned.add(s)
                    remap[e] = s
                    self.last[s] = self.tick
                    used += 1
            while mi < len(miss) and used < len(self.expert_in):
                e = miss[mi]
                mi += 1
                free = [s for s in range(len(self.expert_in)) if s not in pinned and self.expert_in[s] < 0]
                if free:
                    s = free[0]
                else:
                    cand = [s for s in range(len(self.expert_in)) if s not in pinned]
                    s = min(cand, key=lambda x: (self.last[x], x))
                    self.slot_of[self.expert_in[s]] = -1
                self.expert_in[s], self.slot_of[e] = e, s
                pinned.add(s)
                self.last[s] = self.tick
                remap[e] = s
                loads.append((e, s))
                used += 1
            out.append((remap, loads))
            first = False
            self.tick += 1
        return out


@pytest.mark.parametrize("seed", range(8))
def test_slot_cache_matches_model(seed):
    rng = random.Random(seed)
    E, S = rng.choice([(16, 4), (64, 12), (160, 40), (8, 8)])
    c, m = rt.ExpertSlotCache(E, S), _PyCache(E, S)
    for _ in range(60):
        needed = rng.sample(range(E), rng.randint(0, min(E, 3 * S)))
        got = [(list(r), [tuple(x) for x in l]) for r, l in c.plan(needed)]
        assert got == m.plan(needed)
        covered = []
        for remap, loads in got:
            in_pass = [e for e in range(E) if remap[e] >= 0]
            assert len(in_pass) <= S and len({remap[e] for e in in_pass}) == len(in_pass)
            covered += in_pass
        assert sorted(covered) == sorted(set(needed))
        for s in range(S):
            e = c.expert_in(s)
            assert e < 0 or c.slot_of(e) == s
    st = c.stats()
    assert st["hits"] + st["misses"] > 0 and st["passes"] >= 60


def test_resident_experts_are_not_reloaded():
    c = rt.ExpertSlotCache(10, 4)
    (_, loads), = c.plan([1, 2, 3])
    assert sorted(loads) == [(1, 0), (2, 1), (3, 2)]
    (remap, loads), = c.plan([2, 3, 7])
    assert loads == [(7, 3)] and remap[2] == 1 and remap[3] == 2
    assert c.stats()["hits"] == 2
    passes = c.plan([])
    assert len(passes) == 1 and passes[0][1] == []
    with pytest.raises(Exception):
        c.plan([10])


def _fake_weight(E, n, k, seed):
    from rocket_b200.ops import NvFp4Weight
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(0, 256, (E * n, k // 2), generator=g, dtype=torch.uint8)
    sf = torch.randint(0, 256, (E * (n // 128) * (k // 64) * 512,), generator=g, dtype=torch.uint8)
    gs = torch.rand(E * n, generator=g)
    return NvFp4Weight(packed, sf, gs, n, k, E)


def test_streamer_fills_slots_and_rewrites_ids():
    import types

    from rocket_b200.models.expert_stream import ExpertStreamer
    R, n_sh, S, n, k = 12, 1, 3, 128, 128
    w13, w2 = _fake_weight(R + n_sh, 2 * n, k, 1), _fake_weight(R + n_sh, n, 2 * n, 2)
    ref13, ref2 = [t.clone() for t in (w13.packed, w13.sf, w13.gscale)], [t.clone() for t in (w2.packed, w2.sf)]
    L = types.SimpleNamespace(w13=w13, w2=w2, moe=True)
    st = ExpertStreamer(R, n_sh, S, torch.device("cpu"))
    st.adopt(L)
    assert L.w13.num_experts == S + n_sh and L.w2.num_experts == S + n_sh
    pk13, sf13 = 2 * n * k // 2, ref13[1].numel() // (R + n_sh)
    # the shared expert sits after the slots
    assert torch.equal(L.w13.packed.view(-1)[S * pk13:], ref13[0].view(-1)[R * pk13:])
    ids = torch.tensor([[0, 5, R], [5, 7, R], [11, 2, -1], [9, 0, R]], dtype=torch.int32)
    seen = {}
    n_pass = 0
    for i, got in enumerate(st.passes(L, ids)):
        # the slot contents as of this pass (later passes overwrite slots)
        n_pass += 1
        for r in range(ids.shape[0]):
            for j in range(ids.shape[1]):
                e, s = int(ids[r, j]), int(got[r, j])
                if e < 0:
                    assert s == -1
                elif e == R:
                    assert s == (S if i == 0 else -1)
                elif s >= 0:
                    assert torch.equal(L.w13.packed.view(-1)[s * pk13:(s + 1) * pk13],
                                       ref13[0].view(-1)[e * pk13:(e + 1) * pk13])
                    assert torch.equal(L.w13.sf.view(-1)[s * sf13:(s + 1) * sf13],
                                       ref13[1].view(-1)[e * sf13:(e + 1) * sf13])
                    assert torch.equal(L.w13.gscale[s * 2 * n:(s + 1) * 2 * n], ref13[2][e * 2 * n:(e + 1) * 2 * n])
                    seen.setdefault((r, j), []).append(i)
    assert n_pass == 2  # 6 distinct routed experts over 3 slots
    # every routed (token, k) entry runs in exactly one pass
    routed = [(r, j) for r in range(ids.shape[0]) for j in range(ids.shape[1]) if 0 <= int(ids[r, j]) < R]
    assert sorted(seen) == sorted(routed) and all(len(v) == 1 for v in seen.values())
    s = st.stats()
    assert s["misses"] == 6 and s["passes"] == 2 and s["bytes_loaded"] > 0
