"""C++ paged KV manager: refcounts, prefix reuse, fork copy-on-extend, truncate,
eviction safety (reference: engines/glm5-moe-nvfp4-2b/tests/test_kv_radix.cu:1-30)."""
import numpy as np
import pytest

rt = pytest.importorskip("rocket_b200._rt")


def test_append_slots_and_block_table():
    k = rt.KvManager(16, 4, 8, False)
    assert k.open(1, [9] * 10) == 0
    s = k.append(1, list(range(10)))
    pages = k.pages(1)
    assert len(pages) == 3
    assert s == [pages[i // 4] * 4 + i % 4 for i in range(10)]
    bt = np.zeros((1, 8), dtype=np.int32)
    k.block_table([1], bt)
    assert bt[0, :3].tolist() == pages and bt[0, 3:].sum() == 0
    k.free(1)
    assert k.num_free_pages() == 16


def test_prefix_reuse_leaves_one_token_and_refcounts():
    k = rt.KvManager(16, 4, 8, True)
    toks = list(range(12))
    k.open(1, toks)
    k.append(1, toks)
    k.commit_prefix(1)
    assert k.cached_blocks() == 3
    # same 12 tokens: at most 8 reusable (>=1 token must be computed)
    assert k.open(2, toks) == 8
    assert k.pages(2) == k.pages(1)[:2]
    k.free(1)
    k.free(2)
    # cached pages are evictable but still findable
    assert k.num_free_pages() == 16
    assert k.open(3, toks + [99]) == 12


def test_eviction_drops_index_entries():
    k = rt.KvManager(4, 4, 8, True)
    k.open(1, list(range(8)))
    k.append(1, list(range(8)))
    k.commit_prefix(1)
    k.free(1)
    k.open(2, [50 + i for i in range(16)])
    k.append(2, [50 + i for i in range(16)])  # needs all 4 pages -> evicts both cached
    assert k.cached_blocks() == 0
    k.free(2)
    assert k.open(3, list(range(8)) + [1]) == 0


def test_fork_shares_full_pages_and_copies_boundary():
    k = rt.KvManager(16, 4, 8, False)
    k.open(1, [])
    k.append(1, list(range(6)))
    ops = k.fork(1, 2)
    p1, p2 = k.pages(1), k.pages(2)
    assert p1[0] == p2[0] and p1[1] != p2[1]
    assert [(o.src, o.dst) for o in ops] == [(p1[1], p2[1])]
    k.append(2, [7])
    assert k.length(2) == 7 and k.length(1) == 6


def test_truncate_makes_sealed_page_private():
    k = rt.KvManager(16, 4, 8, True)
    toks = list(range(8))
    k.open(1, toks)
    k.append(1, toks)
    k.commit_prefix(1)
    assert k.cached_blocks() == 2
    k.truncate(1, 6)
    assert k.length(1) == 6 and k.cached_blocks() == 1
    k.append(1, [100, 101])
    k.commit_prefix(1)
    assert k.cached_blocks() == 2


def _check_invariants(k, live, ps, total):
    """Structural invariants of the page manager after any operation sequence."""
    owners = {}
    for rid, n in live.items():
        pages = list(k.pages(rid))
        assert k.length(rid) == n
        assert len(pages) == -(-n // ps), (rid, n, pages)
        for p in pages:
            assert 0 <= p < total
            owners.setdefault(p, []).append(rid)
    # the page a sequence writes next (its partial last page) is never shared
    for rid, n in live.items():
        if n % ps:
            last = list(k.pages(rid))[-1]
            assert owners[last] == [rid], (rid, last, owners[last])
    # pages held by live sequences are not free
    assert k.num_free_pages() <= total - len(owners)


def test_random_operations_keep_every_sequences_tokens():
    """Simulated device pages: slots returned by append receive the tokens, copy ops from
    fork / truncate are applied, prefix hits reuse cached pages.  After every operation each
    live sequence must read back exactly its own tokens through its page list."""
    import random
    for seed in range(40):
        rng = random.Random(1000 + seed)
        ps, total = 4, 24
        k = rt.KvManager(total, ps, 16, True)
        mem = [[None] * ps for _ in range(total)]
        live, nxt = {}, 1

        def write(rid, new):
            for slot, tok in zip(k.append(rid, new), new):
                mem[slot // ps][slot % ps] = tok

        def copy(ops):
            for o in ops:
                mem[o.dst] = list(mem[o.src])

        for _ in range(150):
            op = rng.choice(["open", "append", "append", "fork", "truncate", "commit", "free"])
            if op == "open" and len(live) < 5:
                base = rng.choice([[], [1, 2, 3, 4, 5, 6, 7, 8], [1, 2, 3, 4, 9, 9, 9, 9, 5]])
                prompt = base + [rng.randrange(50) for _ in range(rng.randint(1, 6))]
                cached = k.open(nxt, prompt)
                if k.pages_needed(nxt, len(prompt) - cached) > k.num_free_pages():
                    k.free(nxt)
                    continue
                write(nxt, prompt[cached:])
                live[nxt] = list(prompt)
                nxt += 1
            elif op == "append" and live:
                rid = rng.choice(list(live))
                new = [rng.randrange(50) for _ in range(rng.randint(1, 5))]
                if len(live[rid]) + len(new) > 16 * ps or not k.can_append(rid, len(new)):
                    continue
                write(rid, new)
                live[rid] += new
            elif op == "fork" and live and len(live) < 5 and k.num_free_pages() >= 1:
                src = rng.choice(list(live))
                copy(k.fork(src, nxt))
                live[nxt] = list(live[src])
                nxt += 1
            elif op == "truncate" and live:
                rid = rng.choice(list(live))
                n = rng.randint(0, len(live[rid]))
                if k.num_free_pages() < 1:
                    continue
                copy(k.truncate(rid, n))
                live[rid] = live[rid][:n]
            elif op == "commit" and live:
                k.commit_prefix(rng.choice(list(live)))
            elif op == "free" and live:
                rid = rng.choice(list(live))
                k.free(rid)
                del live[rid]
            for rid, toks in live.items():
                pages = list(k.pages(rid))
                got = [mem[pages[i // ps]][i % ps] for i in range(len(toks))]
                assert got == toks, (seed, rid, got, toks)


def test_random_operation_sequences_keep_invariants():
    """Property test: random open / append / fork / truncate / commit / free sequences,
    with prefix caching on, never break the manager's invariants (the reference's radix
    tests cover the same operations one by one, test_kv_radix.cu:1-30)."""
    import random
    for seed in range(40):
        rng = random.Random(seed)
        ps, total = 4, 24
        k = rt.KvManager(total, ps, 16, True)
        live, toks, nxt = {}, {}, 1
        for _ in range(120):
            op = rng.choice(["open", "append", "append", "fork", "truncate", "commit", "free"])
            if op == "open" and len(live) < 5:
                base = rng.choice([[], list(range(rng.randint(1, 12)))])
                prompt = base + [rng.randrange(50) for _ in range(rng.randint(1, 6))]
                cached = k.open(nxt, prompt)
                if k.pages_needed(nxt, len(prompt) - cached) > k.num_free_pages():
                    k.free(nxt)
                    continue
                k.append(nxt, prompt[cached:])
                live[nxt], toks[nxt] = len(prompt), list(prompt)
                nxt += 1
            elif op == "append" and live:
                rid = rng.choice(list(live))
                new = [rng.randrange(50) for _ in range(rng.randint(1, 5))]
                if live[rid] + len(new) > 16 * ps or not k.can_append(rid, len(new)):
                    continue
                k.append(rid, new)
                live[rid] += len(new)
                toks[rid] += new
            elif op == "fork" and live and len(live) < 5:
                src = rng.choice(list(live))
                if k.num_free_pages() < 1:
                    continue
                k.fork(src, nxt)
                live[nxt], toks[nxt] = live[src], list(toks[src])
                nxt += 1
            elif op == "truncate" and live:
                rid = rng.choice(list(live))
                n = rng.randint(0, live[rid])
                k.truncate(rid, n)
                live[rid], toks[rid] = n, toks[rid][:n]
            elif op == "commit" and live:
                k.commit_prefix(rng.choice(list(live)))
            elif op == "free" and live:
                rid = rng.choice(list(live))
                k.free(rid)
                del live[rid], toks[rid]
            _check_invariants(k, live, ps, total)
        for rid in list(live):
            k.free(rid)
        assert k.num_free_pages() == total and k.num_seqs() == 0
