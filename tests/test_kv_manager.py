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
