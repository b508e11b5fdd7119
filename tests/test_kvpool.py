"""CPU: the native KV page pool and the radix prefix cache over pages.

Prefix-cache cases mirror the reference's own tests in
crates/higgs-engine/src/prompt_cache.rs:313-673.  One deliberate difference:
entries keep whole 16-token pages only, so a stored prefix of length n is kept
(and matched) as floor(n/16)*16 tokens, and prefixes under 16 tokens are not
stored at all (the reference stores them but never matches them).
"""
import numpy as np
import pytest

from higgs_b200.ffi import HiggsError
from higgs_b200.kv import BlockPool, PrefixCache


def toks(a, b):
    return np.arange(a, b, dtype=np.int32)


def store(pc, pool, tokens):
    """Store a prefix the way the engine does: the caller owns pages, the cache retains them."""
    n = len(tokens) // 16
    pages = pool.alloc(max(n, 0)) if n else np.zeros(0, np.int32)
    pc.store(tokens, pages)
    if n:
        pool.release(pages)  # drop the caller's reference; the cache keeps its own
    return pages


def test_pool_alloc_release_refcounts():
    pool = BlockPool(8)
    a = pool.alloc(5)
    assert pool.num_free == 3 and len(set(a.tolist())) == 5
    with pytest.raises(HiggsError) as e:
        pool.alloc(4)
    assert e.value.code == -7 and pool.num_free == 3  # all-or-nothing
    pool.retain(a[:2])
    assert pool.refcount(int(a[0])) == 2
    pool.release(a)
    assert pool.num_free == 6
    pool.release(a[:2])
    assert pool.num_free == 8
    with pytest.raises(HiggsError):
        pool.release(a[:1])  # not allocated any more


def test_empty_cache_returns_none():
    pool = BlockPool(16)
    pc = PrefixCache(pool, 10)
    assert pc.lookup([1, 2, 3]) [0] == 0 and len(pc) == 0


def test_store_and_find_exact_match():
    pool = BlockPool(64)
    pc = PrefixCache(pool, 10)
    pages = store(pc, pool, toks(0, 32))
    assert len(pc) == 1
    m, got = pc.lookup(np.concatenate([toks(0, 32), [100, 101, 102]]))
    assert m == 32 and got.tolist() == pages.tolist()
    assert pool.refcount(int(pages[0])) == 2  # cache + this lookup
    pool.release(got)


@pytest.mark.parametrize("stored,query", [((0, 32), (100, 132)), ((0, 8), (0, 32))])
def test_no_match(stored, query):
    pool = BlockPool(16)
    pc = PrefixCache(pool, 10)
    store(pc, pool, toks(*stored))
    assert pc.lookup(toks(*query))[0] == 0


def test_lru_eviction_releases_pages():
    pool = BlockPool(16)
    pc = PrefixCache(pool, 2)
    pa = store(pc, pool, toks(0, 32))
    store(pc, pool, toks(100, 132))
    assert len(pc) == 2 and pool.num_free == 12
    store(pc, pool, toks(200, 232))
    assert len(pc) == 2
    assert pc.lookup(np.concatenate([toks(200, 232), [999]]))[0] == 32
    assert pc.lookup(np.concatenate([toks(0, 32), [999]]))[0] == 0  # A was least recently used
    assert pool.refcount(int(pa[0])) == 0


def test_zero_capacity_never_stores():
    pool = BlockPool(8)
    pc = PrefixCache(pool, 0)
    store(pc, pool, toks(0, 32))
    assert len(pc) == 0 and pool.num_free == 8


def test_clear_releases_everything():
    pool = BlockPool(8)
    pc = PrefixCache(pool, 10)
    store(pc, pool, toks(0, 32))
    pc.clear()
    assert len(pc) == 0 and pool.num_free == 8


def test_longest_prefix_wins():
    pool = BlockPool(32)
    pc = PrefixCache(pool, 10)
    store(pc, pool, toks(0, 20))  # kept as 16
    store(pc, pool, toks(0, 50))  # kept as 48
    assert pc.lookup(toks(0, 64))[0] == 48


def test_overwrite_keeps_len_and_uses_latest():
    pool = BlockPool(32)
    pc = PrefixCache(pool, 1)
    store(pc, pool, toks(0, 32))
    p2 = store(pc, pool, toks(0, 32))
    assert len(pc) == 1
    m, got = pc.lookup(np.concatenate([toks(0, 32), [999]]))
    assert m == 32 and got.tolist() == p2.tolist()


def test_eviction_only_when_new_key():
    pool = BlockPool(32)
    pc = PrefixCache(pool, 2)
    store(pc, pool, toks(0, 32))
    store(pc, pool, toks(100, 132))
    store(pc, pool, toks(0, 32))
    assert len(pc) == 2
    assert pc.lookup(np.concatenate([toks(100, 132), [9]]))[0] == 32
    store(pc, pool, toks(200, 232))
    assert len(pc) == 2
    assert pc.lookup(np.concatenate([toks(200, 232), [9]]))[0] == 32


def test_min_length_boundary():
    pool = BlockPool(8)
    pc = PrefixCache(pool, 10)
    store(pc, pool, toks(0, 16))
    assert pc.lookup(np.concatenate([toks(0, 16), [999]]))[0] == 16
    pc2 = PrefixCache(pool, 10)
    store(pc2, pool, toks(0, 15))
    assert len(pc2) == 0 and pc2.lookup(np.concatenate([toks(0, 15), [999]]))[0] == 0


def test_multiple_overlapping_prefixes():
    pool = BlockPool(64)
    pc = PrefixCache(pool, 10)
    store(pc, pool, toks(0, 16))
    store(pc, pool, toks(0, 32))
    store(pc, pool, toks(0, 64))
    assert len(pc) == 3
    assert pc.lookup(toks(0, 100))[0] == 64
    assert pc.lookup(toks(0, 40))[0] == 32
    assert pc.lookup(toks(0, 20))[0] == 16


def test_shared_prefix_and_diverging_suffixes():
    pool = BlockPool(64)
    pc = PrefixCache(pool, 10)
    store(pc, pool, toks(0, 64))
    store(pc, pool, toks(0, 128))
    q = np.concatenate([toks(0, 64), toks(500, 564)])
    assert pc.lookup(q)[0] == 64
    a = np.concatenate([toks(0, 20), toks(100, 124)])  # 44 -> 32 kept
    b = np.concatenate([toks(0, 20), toks(200, 224)])
    store(pc, pool, a)
    store(pc, pool, b)
    assert pc.lookup(np.concatenate([a, [9]]))[0] == 32
    assert pc.lookup(np.concatenate([b, [9]]))[0] == 32


def test_edge_split_preserves_existing_entry():
    pool = BlockPool(32)
    pc = PrefixCache(pool, 10)
    long_pages = store(pc, pool, toks(0, 50))  # 48 kept
    store(pc, pool, toks(0, 25))  # 16 kept: splits the 48-token edge
    assert len(pc) == 2
    m, got = pc.lookup(np.concatenate([toks(0, 50), [999]]))
    assert m == 48 and got.tolist() == long_pages[:3].tolist()


def test_partial_prefix_served_from_descendant_pages():
    """Beyond the reference (which matches only whole stored prompts): a query sharing the
    first 256 tokens of a stored 512-token prompt reuses its first 16 pages."""
    pool = BlockPool(128)
    pc = PrefixCache(pool, 10)
    rng = np.random.default_rng(2)
    shared = rng.integers(0, 1000, 256).astype(np.int32)
    p1 = np.concatenate([shared, rng.integers(1000, 2000, 256).astype(np.int32)])
    p2 = np.concatenate([shared, rng.integers(2000, 3000, 256).astype(np.int32)])
    pages = store(pc, pool, p1)
    m, got = pc.lookup(p2[:-1])
    assert m == 256 and got.tolist() == pages[:16].tolist()
    assert pool.refcount(int(pages[0])) == 2 and pool.refcount(int(pages[20])) == 1
    pool.release(got)
    # a match ending mid-page is floored to whole pages; under 16 tokens nothing
    q = np.concatenate([p1[:40], [5000]])
    assert pc.lookup(q)[0] == 32
    pool.release(pc.lookup(q)[1])
    assert pc.lookup(np.concatenate([p1[:10], [5000]]))[0] == 0
    # after storing p2 the split node serves p3 as well
    store(pc, pool, p2)
    p3 = np.concatenate([shared, [7, 8, 9]])
    m3, g3 = pc.lookup(p3)
    assert m3 == 256
    pool.release(g3)
